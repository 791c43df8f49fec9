// extern "C" entry points of libkappa_w8 (declared in include/kappa_w8.h).
#include <atomic>
#include <climits>
#include <cmath>

#include "gemm_stream.cuh"
#include "gemm_tc.cuh"
#include "moe.cuh"
#include "norm.cuh"
#include "quant.cuh"

namespace kw8 {
const char* last_error();
void clear_error();
int read_device_status(int32_t* out, cudaStream_t stream);

namespace {

std::atomic<int> g_opt_path{0};        // 0 auto, 1 tensor core, 2 weight streaming
std::atomic<int> g_opt_token_tile{0};  // 0 auto, else 16..256 (multiple of 16)
std::atomic<int> g_opt_deterministic{0};  // 1: MoE combine in a fixed order

// Carves 256-byte aligned sub-buffers out of the caller's workspace.  With
// base == nullptr it only measures.
struct Carver {
  uint8_t* base;
  size_t cap;
  size_t off = 0;
  bool ok = true;
  Carver(void* b, size_t c) : base(static_cast<uint8_t*>(b)), cap(c) {}
  template <class T>
  T* take(int64_t count) {
    const size_t a = (off + 255) & ~static_cast<size_t>(255);
    const size_t need = a + static_cast<size_t>(count < 0 ? 0 : count) * sizeof(T);
    off = need;
    if (base == nullptr) return nullptr;
    if (need > cap) {
      ok = false;
      return nullptr;
    }
    return reinterpret_cast<T*>(base + a);
  }
};

int round16(int64_t v) { return static_cast<int>((v + 15) & ~int64_t(15)); }

// Token tile for the grouped tensor-core path, for groups of mean m routed
// rows (spread about sqrt(m)).
//
// First choice: a group's rows up to m + 3 sqrt(m) split into j near-equal
// tiles of at most kTcMaxDoubleBufferNT rows (the widest tile with two TMEM
// accumulators): nt = that bound / j, rounded up to 16.  It is overruled
// when an expected-cost estimate is at least 20% lower for another tile:
// with R ~ normal(m, sqrt(m)) a group needs E[ceil(R / nt)] = sum_j
// P(R > j nt) tiles, each costing about max(nt, 112) (an MMA below N = 112
// costs the same as at 112).  Measured: at 128 rows per expert (the
// Qwen3-235B-shaped layer, T = 2048) the first choice is 96-row tiles,
// 1446 us, the estimate's 144-row tiles 954 us; at 256 rows per expert the
// first choice (160) is 2.5% faster than the estimate's 144 (which it
// rates 9% cheaper: hence the 20% bar).
double expected_tile_cost(double m, int nt) {
  const double sd = std::sqrt(std::max(m, 1.0));
  double tiles = 0.0;
  for (int j = 0; j * nt < m + 8.0 * sd + nt; ++j)
    tiles += 0.5 * std::erfc((j * nt - m) / (sd * std::sqrt(2.0)));
  return tiles * std::max(nt, 112);
}

int pick_nt(int64_t rows, int64_t groups) {
  const int forced = g_opt_token_tile.load();
  if (forced >= 16 && forced <= kTcMaxNT && forced % 16 == 0) return forced;
  const double m = static_cast<double>(rows) / static_cast<double>(groups > 0 ? groups : 1);
  const double hi = m + 3.0 * std::sqrt(m);
  const int64_t j = std::max<int64_t>(1, static_cast<int64_t>(std::ceil(hi / kTcMaxDoubleBufferNT)));
  int64_t first = round16(static_cast<int64_t>(std::ceil(hi / static_cast<double>(j))));
  first = std::min<int64_t>(std::max<int64_t>(first, 16), kTcMaxDoubleBufferNT);
  int best = static_cast<int>(first);
  double best_cost = expected_tile_cost(m, best);
  const double bar = 0.8 * best_cost;
  for (int nt = 16; nt <= kTcMaxDoubleBufferNT; nt += 16) {
    const double cost = expected_tile_cost(m, nt);
    if (cost <= bar && cost < best_cost) {
      best_cost = cost;
      best = nt;
    }
  }
  return best;
}

// Token tile for a dense (single-group) tensor-core GEMM with `m_tiles`
// feature tiles: the fewest waves over the SMs times a tile's cost.  A
// tcgen05.mma (M = 128, K = 16) costs its issuing thread about the same
// ~130-160 cycles for any N up to 256, so a tile's cost hardly depends on
// its rows; what does: 160-row tiles hold fewer pipeline stages than
// 128-row ones (cost ~ max(128, nt) up to 160, measured), and a 192-row
// tile (one TMEM accumulator, three stages, five A slots) costs about 6%
// more than a 128-row one.  Wider tiles keep only two stages and are not
// taken.  Measured on the Gemma3-4B MLP: T = 256 -> 128-row tiles (82 us;
// 192: 92 us), T = 512 -> 192-row tiles (118 us; 128: 139 us).  Ties go to
// the larger tile.
int pick_nt_dense(int64_t rows, int64_t m_tiles) {
  const int forced = g_opt_token_tile.load();
  if (forced >= 16 && forced <= kTcMaxNT && forced % 16 == 0) return forced;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  const int64_t sms = num_sms(dev);
  int best = 16;
  int64_t best_cost = INT64_MAX;
  for (int nt = 16; nt <= 192; nt += 16) {
    if (nt > kTcMaxDoubleBufferNT && nt != 192) continue;
    const int64_t tiles = (rows + nt - 1) / nt * m_tiles;
    const int64_t waves = (tiles + sms - 1) / sms;
    const int64_t cost = waves * (nt == 192 ? 136 : (nt > 128 ? nt : 128));
    if (cost < best_cost || (cost == best_cost && nt > best)) {
      best = nt;
      best_cost = cost;
    }
    if (nt >= rows) break;
  }
  return best;
}

// K splits for a dense tensor-core GEMM of `tiles` output tiles over
// k_tiles k tiles: split only when the tiles fill at most half the SMs,
// into at most 8 ranges of at least 4 k tiles, filling the SMs once
// (fp32 partials, summed in range order by launch_reduce_splits).
int pick_k_splits(int64_t tiles, int64_t k_tiles) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  const int64_t sms = num_sms(dev);
  if (tiles <= 0 || tiles * 2 > sms) return 1;
  const int64_t want = std::min<int64_t>({sms / tiles, k_tiles / 4, 8});
  return valid_k_splits(static_cast<int>(std::max<int64_t>(want, 1)), k_tiles);
}

// Split plan of a dense tensor-core GEMM with fp32 output: T rows, N_out
// features (128 per tile), K; 1 = no split.
int dense_f32_splits(int64_t T, int64_t N_out, int64_t K) {
  const int64_t m_tiles = (N_out + 127) / 128;
  const int nt = pick_nt_dense(T, m_tiles);
  return pick_k_splits((T + nt - 1) / nt * m_tiles, (K + kTcBK - 1) / kTcBK);
}

// Router logits on the tensor-core path (T above kStreamRouterMaxRows) with
// a split: the fp32 partial buffer it needs, in floats (0 without split).
int64_t router_part_floats(int64_t T, int64_t D, int64_t E);

// Routed rows per group up to m + 3 sqrt(m) for groups of mean m rows.
double rows_hint(int64_t rows, int64_t groups) {
  const double mean = static_cast<double>(rows) / static_cast<double>(groups > 0 ? groups : 1);
  return mean + 3.0 * std::sqrt(mean);
}

// Weight-streaming kernel (gemm_stream) instead of the tensor-core pipeline
// when a group's rows fit a pass of at most 16 rows: the work is then bound
// by weight bytes, and the tensor-core pipeline's per-stage cost (one
// mbarrier round trip and eight MMAs of N <= 32 per 16 KB of weights) caps
// it well below HBM bandwidth.  Measured on the Qwen3-30B-A3B layer: the
// streaming kernel is faster up to 64 decode tokens (<= 16 rows per expert;
// 173 vs 221 us at 64), the tensor-core pipeline from 128 (224 vs 297 us).
constexpr double kStreamMaxRowsHint = 16.0;

bool use_stream(double hint) {
  const int p = g_opt_path.load();
  if (p == 1) return false;
  if (p == 2) return true;
  return hint <= kStreamMaxRowsHint;
}

constexpr int kStreamMaxKz = 16;  // CTAs sharing a feature tile's K, weight-streaming path

// Router logits: dense rows of the router GEMM up to this many go to the
// weight-streaming kernel.
constexpr int64_t kStreamRouterMaxRows = 256;

int check_weight(const kw8_weight& w, const char* name) {
  KW8_REQUIRE(w.q != nullptr && w.scale != nullptr, KW8_ERR_INVALID_ARG, "%s: null pointer", name);
  KW8_REQUIRE(w.scale_dtype == KW8_DT_F32 || w.scale_dtype == KW8_DT_BF16, KW8_ERR_INVALID_ARG,
              "%s: scale dtype must be f32 or bf16", name);
  KW8_REQUIRE(w.per_channel == 0 || w.per_channel == 1, KW8_ERR_INVALID_ARG,
              "%s: per_channel must be 0 or 1", name);
  KW8_REQUIRE(w.layout == KW8_LAYOUT_KMAJOR || w.layout == KW8_LAYOUT_TILED, KW8_ERR_INVALID_ARG,
              "%s: unknown layout %d", name, w.layout);
  KW8_REQUIRE(w.layout == KW8_LAYOUT_KMAJOR || (reinterpret_cast<uintptr_t>(w.q) & 15) == 0,
              KW8_ERR_UNSUPPORTED, "%s: tiled weights must be 16-byte aligned", name);
  return KW8_OK;
}

// Paired gate/up weights are read by one kernel: one layout for both.
int check_same_layout(const kw8_weight& a, const kw8_weight& b) {
  KW8_REQUIRE(a.layout == b.layout, KW8_ERR_INVALID_ARG, "gate and up weights must share one layout");
  return KW8_OK;
}

GemmArgs base_args(const kw8_weight& a, const kw8_weight* b) {
  GemmArgs g{};
  g.a_tiled = a.layout == KW8_LAYOUT_TILED ? 1 : 0;
  g.scale_a = a.scale;
  g.scale_a_dtype = a.scale_dtype;
  g.scale_a_pc = a.per_channel;
  if (b) {
    g.scale_b = b->scale;
    g.scale_b_dtype = b->scale_dtype;
    g.scale_b_pc = b->per_channel;
  } else {
    g.scale_b = a.scale;
    g.scale_b_dtype = a.scale_dtype;
    g.scale_b_pc = a.per_channel;
  }
  return g;
}

StreamArgs stream_args(const kw8_weight& a, const kw8_weight* b) {
  StreamArgs g{};
  g.w_tiled = a.layout == KW8_LAYOUT_TILED ? 1 : 0;
  g.scale_a = a.scale;
  g.scale_a_dtype = a.scale_dtype;
  g.scale_a_pc = a.per_channel;
  if (b) {
    g.scale_b = b->scale;
    g.scale_b_dtype = b->scale_dtype;
    g.scale_b_pc = b->per_channel;
  }
  return g;
}

// One grouped GEMM on the tensor-core pipeline.
int run_gemm(int mode, const kw8_weight& a, const kw8_weight* b, int64_t groups, int64_t N_out,
             int64_t K, const void* x, int64_t x_rows, int64_t ldx, const GemmArgs& args,
             cudaStream_t stream) {
  return launch_gemm_tc(mode, a.q, b ? b->q : nullptr, groups, N_out, K, x, x_rows, ldx, args,
                        stream);
}

struct MoeBuffers {
  float* logits;
  int32_t* idx;
  __nv_bfloat16* w;
  int32_t* sorted_token;
  int32_t* inv_pos;
  float* sorted_w;
  int32_t* group_sizes;
  int32_t* group_offsets;
  TileEntry* tiles;
  int32_t* num_tiles;
  __nv_bfloat16* xs;
  __nv_bfloat16* h;
  float* acc;  // [T][D] fp32 accumulation of the fused combine
  int32_t* perm_hist;  // per-block expert histograms of the permutation
  int32_t* active;     // [E + 1]: count, then the experts that kept rows
  float* router_part;  // split-K partial logits of the tensor-core router (or empty)
};

struct ExpertBuffers {
  TileEntry* tiles;
  int32_t* num_tiles;
  __nv_bfloat16* h;
};

int64_t tile_capacity(int64_t rows, int64_t groups, int nt_min) {
  return groups + (rows + nt_min - 1) / nt_min + 1;
}

ExpertBuffers carve_expert(Carver& c, int64_t rows, int64_t I, int64_t E) {
  ExpertBuffers b;
  b.tiles = c.take<TileEntry>(tile_capacity(rows, E, 8));
  b.num_tiles = c.take<int32_t>(1);
  b.h = c.take<__nv_bfloat16>(rows * I);
  return b;
}

MoeBuffers carve_moe(Carver& c, int64_t T, int64_t D, int64_t I, int64_t E, int k) {
  MoeBuffers b;
  const int64_t m = T * k;
  b.logits = c.take<float>(T * E);
  b.idx = c.take<int32_t>(m);
  b.w = c.take<__nv_bfloat16>(m);
  b.sorted_token = c.take<int32_t>(m);
  b.inv_pos = c.take<int32_t>(m);
  b.sorted_w = c.take<float>(m);
  b.group_sizes = c.take<int32_t>(E);
  b.group_offsets = c.take<int32_t>(E + 1);
  b.tiles = c.take<TileEntry>(tile_capacity(m, E, 8));
  b.num_tiles = c.take<int32_t>(1);
  b.xs = c.take<__nv_bfloat16>(m * D);
  b.h = c.take<__nv_bfloat16>(m * I);
  b.acc = c.take<float>(T * D);
  b.router_part = c.take<float>(router_part_floats(T, D, E));
  b.perm_hist = c.take<int32_t>(permute_hist_ints(E));
  b.active = c.take<int32_t>(E + 1);
  return b;
}

// Expert FFN over rows sorted by group (gate/up + SwiGLU, down).  Row r of
// the sorted order is x row `row_index[r]` (weight-streaming path only: the
// gather is fused into its operand load) or, with row_index == nullptr, x
// row r.  With row_token / row_weight the down projection runs the fused
// combine (EPI_COMBINE_F32) into `ys` = fp32 [T][D] accumulation buffer;
// otherwise `ys` is bf16 [rows][D].
int expert_ffn(bool streamed, const void* x, const int32_t* row_index, int64_t rows, int64_t D,
               int64_t I, int64_t E, const int32_t* group_offsets, const kw8_weight& gate,
               const kw8_weight& up, const kw8_weight& down, void* ys, const ExpertBuffers& b,
               cudaStream_t stream, const int32_t* row_token = nullptr,
               const float* row_weight = nullptr, const int32_t* active = nullptr,
               int64_t tile_rows = -1) {
  // tile_rows: the rows the E groups hold together, for the tile choice,
  // when `rows` (the extent of the row buffers) counts other groups' rows too.
  const int64_t hint = tile_rows >= 0 ? tile_rows : rows;
  const int mode = row_token != nullptr ? EPI_COMBINE_F32 : EPI_PLAIN_BF16;
  if (int rc = check_same_layout(gate, up)) return rc;
  if (streamed) {
    const int nt = stream_nt(rows_hint(hint, E));
    StreamArgs g = stream_args(gate, &up);
    g.group_offsets = group_offsets;
    g.active_groups = active;
    g.row_index = row_index;
    g.out = b.h;
    g.ld_out = I;
    int rc = launch_gemm_stream(EPI_PAIR_SILU, gate.q, up.q, E, I, D, x, D, hint, nt, g, stream);
    if (rc) return rc;
    StreamArgs d = stream_args(down, nullptr);
    d.group_offsets = group_offsets;
    d.active_groups = active;
    d.out = ys;
    d.ld_out = D;
    d.row_token = row_token;
    d.row_weight = row_weight;
    d.kz_max = kStreamMaxKz;  // used by the combine mode only (its atomics add the K ranges)
    return launch_gemm_stream(mode, down.q, nullptr, E, D, I, b.h, I, hint, nt, d, stream);
  }
  KW8_REQUIRE(row_index == nullptr, KW8_ERR_INVALID_ARG, "tensor-core path takes gathered rows");
  const int nt = pick_nt(hint, E);
  int rc = launch_build_tiles(group_offsets, E, nt, b.tiles, b.num_tiles, stream);
  if (rc) return rc;
  GemmArgs g = base_args(gate, &up);
  g.tiles = b.tiles;
  g.num_tiles = b.num_tiles;
  g.nt = nt;
  g.out = b.h;
  g.ld_out = I;
  rc = run_gemm(EPI_PAIR_SILU, gate, &up, E, I, D, x, rows, D, g, stream);
  if (rc) return rc;
  GemmArgs d = base_args(down, nullptr);
  d.tiles = b.tiles;
  d.num_tiles = b.num_tiles;
  d.nt = nt;
  d.out = ys;
  d.ld_out = D;
  d.row_token = row_token;
  d.row_weight = row_weight;
  return run_gemm(mode, down, nullptr, E, D, I, b.h, rows, I, d, stream);
}

bool router_streamed(int64_t T) {
  const int path = g_opt_path.load();
  return path == 2 || (path == 0 && T <= kStreamRouterMaxRows);
}

// K split over CTAs of a dense fp32-output weight-streaming GEMM (1: none).
int stream_f32_kz(int64_t T, int64_t N_out, int64_t K) {
  const int nt = stream_nt(static_cast<double>(T));
  return stream_plan(EPI_PLAIN_F32, nt, false, false, 1, T, T, N_out, K, kStreamMaxKz).kz;
}

// K split of the weight-streaming router: none up to 16 tokens, where the
// reduction of the partials cost more than the split saved.
int router_stream_kz(int64_t T, int64_t D, int64_t E) {
  return T <= 16 ? 1 : stream_f32_kz(T, E, D);
}

// Sized for the larger split of the two paths, so that a workspace sized
// under one GEMM-path option also serves the other.
int64_t router_part_floats(int64_t T, int64_t D, int64_t E) {
  const int splits = std::max(router_stream_kz(T, D, E), dense_f32_splits(T, E, D));
  return splits > 1 ? splits * T * E : 0;
}

// Router logits [T][E] fp32.  `part` (router_part_floats(T, D, E) floats,
// or nullptr) lets the GEMM split K over more SMs.
int router_logits(const void* x, int64_t T, int64_t D, int64_t E, const kw8_weight& router,
                  float* logits, cudaStream_t stream, float* part = nullptr) {
  int rc;
  if (router_streamed(T)) {
    StreamArgs r = stream_args(router, nullptr);
    r.dense_rows = static_cast<int>(T);
    r.out = logits;
    r.ld_out = E;
    const int kz = part != nullptr ? router_stream_kz(T, D, E) : 1;
    if (kz > 1) {
      r.out = part;
      r.kz_max = kStreamMaxKz;
      r.split_stride = T * E;
    }
    rc = launch_gemm_stream(EPI_PLAIN_F32, router.q, nullptr, 1, E, D, x, D, T,
                            stream_nt(static_cast<double>(T)), r, stream);
    if (!rc && kz > 1) rc = launch_reduce_splits(part, kz, T * E, T * E, logits, false, stream);
  } else {
    GemmArgs r = base_args(router, nullptr);
    r.dense_rows = static_cast<int>(T);
    r.nt = pick_nt_dense(T, (E + 127) / 128);
    r.out = logits;
    r.ld_out = E;
    const int splits = part != nullptr ? dense_f32_splits(T, E, D) : 1;
    if (splits > 1) {
      r.out = part;
      r.k_splits = splits;
      r.split_stride = T * E;
    }
    rc = run_gemm(EPI_PLAIN_F32, router, nullptr, 1, E, D, x, T, D, r, stream);
    if (!rc && splits > 1) rc = launch_reduce_splits(part, splits, T * E, T * E, logits, false, stream);
  }
  return rc;
}

// Router logits + top-k (zero_rows: see launch_topk).
int route(const void* x, int64_t T, int64_t D, int64_t E, int k, const kw8_weight& router,
          float* logits, int32_t* idx, void* w, cudaStream_t stream, float* part = nullptr,
          float* zero_rows = nullptr, int64_t zero_cols = 0) {
  const int rc = router_logits(x, T, D, E, router, logits, stream, part);
  if (rc) return rc;
  return launch_topk(logits, T, E, k, idx, w, stream, zero_rows, zero_cols);
}

// K split of the dense down projection on the path the option selects (1:
// none), and its fp32 partials sized for the larger split of the two paths
// (a workspace sized under one option also serves the other).
int dense_down_splits(int64_t T, int64_t D, int64_t H) {
  if (T <= 0) return 1;
  return use_stream(static_cast<double>(T)) ? stream_f32_kz(T, D, H) : dense_f32_splits(T, D, H);
}

int64_t dense_down_part_floats(int64_t T, int64_t D, int64_t H) {
  if (T <= 0) return 0;
  const int splits = std::max(stream_f32_kz(T, D, H), dense_f32_splits(T, D, H));
  return splits > 1 ? splits * T * D : 0;
}

// Gate/up GEMM with the activation epilogue: h [T][H] bf16.
int dense_gate_up(const void* x, int64_t T, int64_t D, int64_t H, const kw8_weight& gate,
                  const kw8_weight& up, int act, __nv_bfloat16* h, cudaStream_t stream) {
  if (int rc = check_same_layout(gate, up)) return rc;
  const int epi_pair = act == KW8_ACT_GELU_TANH ? EPI_PAIR_GELU : EPI_PAIR_SILU;
  if (use_stream(static_cast<double>(T))) {
    StreamArgs g = stream_args(gate, &up);
    g.dense_rows = static_cast<int>(T);
    g.out = h;
    g.ld_out = H;
    return launch_gemm_stream(epi_pair, gate.q, up.q, 1, H, D, x, D, T, stream_nt(static_cast<double>(T)), g,
                              stream);
  }
  GemmArgs g = base_args(gate, &up);
  g.dense_rows = static_cast<int>(T);
  g.nt = pick_nt_dense(T, (H + 63) / 64);
  g.out = h;
  g.ld_out = H;
  return run_gemm(epi_pair, gate, &up, 1, H, D, x, T, D, g, stream);
}

// A dense W8 product y = x . w^T (x [T][K] bf16 -> [T][N]) as fp32 partial
// sums part[s][T][N], s < splits (1: one slice), on the path the option
// selects; `splits` comes from linear_splits().
int dense_f32_parts(const void* x, int64_t T, int64_t K, int64_t N, const kw8_weight& w, int splits,
                    float* part, cudaStream_t stream) {
  if (use_stream(static_cast<double>(T))) {
    StreamArgs d = stream_args(w, nullptr);
    d.dense_rows = static_cast<int>(T);
    d.out = part;
    d.ld_out = N;
    if (splits > 1) {
      d.kz_max = kStreamMaxKz;
      d.split_stride = T * N;
    }
    return launch_gemm_stream(EPI_PLAIN_F32, w.q, nullptr, 1, N, K, x, K, T, stream_nt(static_cast<double>(T)), d,
                              stream);
  }
  GemmArgs d = base_args(w, nullptr);
  d.dense_rows = static_cast<int>(T);
  d.nt = pick_nt_dense(T, (N + 127) / 128);
  d.out = part;
  d.ld_out = N;
  if (splits > 1) {
    d.k_splits = splits;
    d.split_stride = T * N;
  }
  return run_gemm(EPI_PLAIN_F32, w, nullptr, 1, N, K, x, T, K, d, stream);
}

// ------------------------------------------------------- W8 linear ----

// A linear layer takes the weight-streaming kernel for few rows, or when
// its output is narrow (at most two 128-feature tiles: the tensor-core
// kernel would keep few SMs busy) up to kStreamRouterMaxRows rows.
bool linear_streamed(int64_t T, int64_t N) {
  const int path = g_opt_path.load();
  if (path != 0) return path == 2;
  return T <= static_cast<int64_t>(kStreamMaxRowsHint) || (N <= 256 && T <= kStreamRouterMaxRows);
}

// K split of a linear layer on its path (1: none).
int linear_splits(int64_t T, int64_t K, int64_t N) {
  return linear_streamed(T, N) ? stream_f32_kz(T, N, K) : dense_f32_splits(T, N, K);
}

struct LinearBuffers {
  __nv_bfloat16* xg;  // gathered rows (tensor-core path with a row index)
  float* part;        // split-K partial sums
};

LinearBuffers carve_linear(Carver& c, int64_t T, int64_t K, int64_t N) {
  LinearBuffers b;
  b.xg = c.take<__nv_bfloat16>(T * K);
  const int splits = std::max(stream_f32_kz(T, N, K), dense_f32_splits(T, N, K));
  b.part = c.take<float>(splits > 1 ? splits * T * N : 0);
  return b;
}

int linear(const void* x, const int32_t* rows, int64_t T, int64_t K, int64_t N, const kw8_weight& w,
           bool out_f32, void* out, const LinearBuffers& b, cudaStream_t stream) {
  const bool streamed = linear_streamed(T, N);
  const int splits = linear_splits(T, K, N);
  const int mode = out_f32 ? EPI_PLAIN_F32 : EPI_PLAIN_BF16;
  if (streamed) {
    StreamArgs a = stream_args(w, nullptr);
    a.dense_rows = static_cast<int>(T);
    a.row_index = rows;  // the gather is fused into the operand load
    a.out = out;
    a.ld_out = N;
    if (splits > 1) {
      a.out = b.part;
      a.kz_max = kStreamMaxKz;
      a.split_stride = T * N;
    }
    int rc = launch_gemm_stream(splits > 1 ? EPI_PLAIN_F32 : mode, w.q, nullptr, 1, N, K, x, K, T,
                                stream_nt(static_cast<double>(T)), a, stream);
    if (rc || splits <= 1) return rc;
    return launch_reduce_splits(b.part, splits, T * N, T * N, out, !out_f32, stream);
  }
  const void* xs = x;
  if (rows != nullptr) {
    // The TMA loads need the rows contiguous: gather them first.
    int rc = launch_gather(x, rows, nullptr, T, K, b.xg, stream);
    if (rc) return rc;
    xs = b.xg;
  }
  GemmArgs a = base_args(w, nullptr);
  a.dense_rows = static_cast<int>(T);
  a.nt = pick_nt_dense(T, (N + 127) / 128);
  a.out = out;
  a.ld_out = N;
  if (splits > 1) {
    a.out = b.part;
    a.k_splits = splits;
    a.split_stride = T * N;
  }
  int rc = run_gemm(splits > 1 ? EPI_PLAIN_F32 : mode, w, nullptr, 1, N, K, xs, T, K, a, stream);
  if (rc || splits <= 1) return rc;
  return launch_reduce_splits(b.part, splits, T * N, T * N, out, !out_f32, stream);
}

int check_moe_args(int64_t T, int64_t D, int64_t I, int64_t E, int k, const kw8_weight& router,
                   const kw8_weight& gate, const kw8_weight& up, const kw8_weight& down) {
  KW8_REQUIRE(T >= 0 && D > 0 && I > 0 && E > 0 && k >= 1 && k <= E, KW8_ERR_INVALID_ARG,
              "bad shape (T=%lld D=%lld I=%lld E=%lld k=%d)", (long long)T, (long long)D,
              (long long)I, (long long)E, k);
  int rc = check_weight(router, "router");
  if (!rc) rc = check_weight(gate, "gate");
  if (!rc) rc = check_weight(up, "up");
  if (!rc) rc = check_weight(down, "down");
  if (rc) return rc;
  KW8_REQUIRE(T * k < (1ll << 31), KW8_ERR_UNSUPPORTED, "too many routed rows");
  return KW8_OK;
}

// The MoE layer up to its fp32 output b.acc [T][D] (T >= 1).
int moe_layer_acc(const void* x, int64_t T, int64_t D, int64_t I, int64_t E, int k, int64_t capacity,
                  const kw8_weight& router, const kw8_weight& gate, const kw8_weight& up,
                  const kw8_weight& down, const MoeBuffers& b, cudaStream_t stream) {
  const int64_t m = T * k;
  int rc;
  // The top-k kernel also zeroes the fp32 combine buffer (one row per token).
  float* part = router_part_floats(T, D, E) > 0 ? b.router_part : nullptr;
  if (route_tail_small_ok(T, E, k)) {  // decode: top-k, permutation and zeroing in one launch
    rc = router_logits(x, T, D, E, router, b.logits, stream, part);
    if (!rc)
      rc = launch_route_tail_small(b.logits, T, E, k, capacity, b.idx, b.w, b.sorted_token,
                                   b.inv_pos, b.group_sizes, b.group_offsets, b.sorted_w,
                                   b.active, b.acc, D, stream);
  } else {
    rc = kw8::route(x, T, D, E, k, router, b.logits, b.idx, b.w, stream, part, b.acc, D);
    if (!rc)
      rc = launch_permute_multi(b.idx, T, k, E, capacity, b.perm_hist, b.sorted_token, b.inv_pos,
                                b.group_sizes, b.group_offsets, stream, b.w, b.sorted_w, b.active);
  }
  if (rc) return rc;
  // Few rows per expert: the weight-streaming kernels read x rows through
  // the permutation (no gathered copy); otherwise gather for the TMA loads.
  const bool streamed = use_stream(rows_hint(m, E));
  if (!streamed) {
    rc = launch_gather(x, b.sorted_token, b.group_offsets + E, m, D, b.xs, stream);
    if (rc) return rc;
  }
  ExpertBuffers eb{b.tiles, b.num_tiles, b.h};
  if (g_opt_deterministic.load()) {
    // Deterministic combine: the expert outputs are stored as bf16 rows in
    // sorted order (into xs, free once gate/up has read it; kappa also
    // rounds them to bf16, ffn_moe.py:213) and each token's k rows are
    // summed in slot order.
    rc = expert_ffn(streamed, streamed ? x : b.xs, streamed ? b.sorted_token : nullptr, m, D, I, E,
                    b.group_offsets, gate, up, down, b.xs, eb, stream, nullptr, nullptr, b.active);
    if (rc) return rc;
    return launch_combine(b.xs, b.inv_pos, b.w, T, k, D, b.acc, stream, true);
  }
  // The down projection adds w * y of every routed row straight into the
  // fp32 token buffer (zeroed by the top-k kernel; no bf16 rounding of the
  // per-expert outputs, no [T*k][D] round trip).  The order of those fp32
  // additions varies from call to call.
  return expert_ffn(streamed, streamed ? x : b.xs, streamed ? b.sorted_token : nullptr, m, D, I, E,
                    b.group_offsets, gate, up, down, b.acc, eb, stream, b.sorted_token, b.sorted_w,
                    b.active);
}

int check_norms(const kw8_block_norms* n, int64_t D) {
  KW8_REQUIRE(n != nullptr && n->pre_scale != nullptr, KW8_ERR_INVALID_ARG, "block norms: pre-FFN scale required");
  (void)D;
  return KW8_OK;
}

}  // namespace
}  // namespace kw8

using namespace kw8;

#define KW8_API_BEGIN clear_error();

extern "C" {

const char* kw8_last_error(void) { return kw8::last_error(); }

int32_t kw8_abi_version(void) { return 3; }

int kw8_device_status(int32_t* status_out, kw8_stream_t stream) {
  KW8_API_BEGIN
  return read_device_status(status_out, stream);
}

int kw8_set_option(int32_t option, int64_t value) {
  KW8_API_BEGIN
  if (option == 0) {
    KW8_REQUIRE(value >= 0 && value <= 2, KW8_ERR_INVALID_ARG, "path must be 0, 1 or 2");
    g_opt_path.store(static_cast<int>(value));
    return KW8_OK;
  }
  if (option == 1) {
    KW8_REQUIRE(value == 0 || (value >= 16 && value <= kTcMaxNT && value % 16 == 0),
                KW8_ERR_INVALID_ARG, "token tile must be 0 or a multiple of 16 in [16, 256]");
    g_opt_token_tile.store(static_cast<int>(value));
    return KW8_OK;
  }
  if (option == 4) {
    KW8_REQUIRE(value == 0 || value == 1, KW8_ERR_INVALID_ARG, "EP phase timing must be 0 or 1");
    g_opt_ep_timing.store(static_cast<int>(value));
    return KW8_OK;
  }
  if (option == 3) {
    KW8_REQUIRE(value >= 0 && value <= 2, KW8_ERR_INVALID_ARG, "CTA-pair GEMM must be 0, 1 or 2");
    g_opt_tc_pair.store(static_cast<int>(value));
    return KW8_OK;
  }
  if (option == 2) {
    KW8_REQUIRE(value == 0 || value == 1, KW8_ERR_INVALID_ARG, "deterministic must be 0 or 1");
    g_opt_deterministic.store(static_cast<int>(value));
    return KW8_OK;
  }
  return fail(KW8_ERR_INVALID_ARG, "unknown option %d", option);
}

size_t kw8_quantize_workspace_size(int64_t outer, int64_t N) {
  return kw8::quantize_workspace_size(outer, N);
}

int kw8_quantize(const void* w, int32_t w_dtype, int64_t outer, int64_t K, int64_t N,
                 int64_t stride_outer, int64_t stride_k, int64_t stride_n, int32_t per_channel,
                 int32_t scale_dtype, int8_t* q_out, void* scale_out, void* workspace,
                 size_t workspace_bytes, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(per_channel == 0 || per_channel == 1, KW8_ERR_INVALID_ARG, "per_channel must be 0/1");
  return launch_quantize(w, w_dtype, outer, K, N, stride_outer, stride_k, stride_n, per_channel,
                         scale_dtype, q_out, scale_out, workspace, workspace_bytes, stream);
}

int kw8_dequantize(kw8_weight w, int64_t groups, int64_t N, int64_t K, int32_t out_dtype,
                   void* out, kw8_stream_t stream) {
  KW8_API_BEGIN
  int rc = check_weight(w, "weight");
  if (rc) return rc;
  KW8_REQUIRE(w.layout == KW8_LAYOUT_KMAJOR, KW8_ERR_UNSUPPORTED,
              "dequantize takes K-major values (kw8_unpack_weight a tiled weight first)");
  return launch_dequantize(w, groups, N, K, out_dtype, out, stream);
}

size_t kw8_packed_weight_bytes(int64_t groups, int64_t N, int64_t K) {
  if (groups <= 0 || N <= 0 || K <= 0) return 0;
  return static_cast<size_t>(tiled_bytes(groups, N, K));
}

int kw8_pack_weight(const int8_t* q, int64_t groups, int64_t N, int64_t K, void* tiled, kw8_stream_t stream) {
  KW8_API_BEGIN
  return launch_pack(q, groups, N, K, tiled, stream);
}

int kw8_unpack_weight(const void* tiled, int64_t groups, int64_t N, int64_t K, int8_t* q,
                      kw8_stream_t stream) {
  KW8_API_BEGIN
  return launch_unpack(tiled, groups, N, K, q, stream);
}

size_t kw8_dense_ffn_workspace_size(int64_t T, int64_t D, int64_t H) {
  Carver c(nullptr, SIZE_MAX);
  c.take<__nv_bfloat16>(T * H);
  c.take<float>(dense_down_part_floats(T, D, H));
  return c.off;
}

int kw8_dense_ffn(const void* x, int64_t T, int64_t D, int64_t H, kw8_weight gate, kw8_weight up,
                  kw8_weight down, int32_t act, int32_t out_dtype, void* out, void* workspace,
                  size_t workspace_bytes, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(x && out, KW8_ERR_INVALID_ARG, "null x/out");
  KW8_REQUIRE(T >= 0 && D > 0 && H > 0, KW8_ERR_INVALID_ARG, "bad shape");
  KW8_REQUIRE(act == KW8_ACT_GELU_TANH || act == KW8_ACT_SILU, KW8_ERR_INVALID_ARG, "bad act");
  KW8_REQUIRE(out_dtype == KW8_DT_BF16 || out_dtype == KW8_DT_F32, KW8_ERR_INVALID_ARG,
              "bad out dtype");
  int rc = check_weight(gate, "gate");
  if (!rc) rc = check_weight(up, "up");
  if (!rc) rc = check_weight(down, "down");
  if (rc) return rc;
  if (T == 0) return KW8_OK;
  KW8_REQUIRE(T < (1ll << 31), KW8_ERR_UNSUPPORTED, "too many tokens");
  Carver c(workspace, workspace_bytes);
  __nv_bfloat16* h = c.take<__nv_bfloat16>(T * H);
  float* part = c.take<float>(dense_down_part_floats(T, D, H));
  const int splits = dense_down_splits(T, D, H);
  KW8_REQUIRE(workspace != nullptr && c.ok, KW8_ERR_WORKSPACE, "dense FFN workspace too small");
  const int epi_pair = act == KW8_ACT_GELU_TANH ? EPI_PAIR_GELU : EPI_PAIR_SILU;
  const int epi_out = out_dtype == KW8_DT_F32 ? EPI_PLAIN_F32 : EPI_PLAIN_BF16;
  if (use_stream(static_cast<double>(T))) {
    const int nt = stream_nt(static_cast<double>(T));
    StreamArgs g = stream_args(gate, &up);
    g.dense_rows = static_cast<int>(T);
    g.out = h;
    g.ld_out = H;
    rc = launch_gemm_stream(epi_pair, gate.q, up.q, 1, H, D, x, D, T, nt, g, stream);
    if (rc) return rc;
    StreamArgs d = stream_args(down, nullptr);
    d.dense_rows = static_cast<int>(T);
    d.out = out;
    d.ld_out = D;
    if (splits > 1) {
      // Few rows and long K: the CTAs split K into fp32 partials, summed in
      // order into the output.
      const int kz = splits;
      d.out = part;
      d.kz_max = kStreamMaxKz;
      d.split_stride = T * D;
      rc = launch_gemm_stream(EPI_PLAIN_F32, down.q, nullptr, 1, D, H, h, H, T, nt, d, stream);
      if (rc) return rc;
      return launch_reduce_splits(part, kz, T * D, T * D, out, out_dtype == KW8_DT_BF16, stream);
    }
    return launch_gemm_stream(epi_out, down.q, nullptr, 1, D, H, h, H, T, nt, d, stream);
  }
  GemmArgs g = base_args(gate, &up);
  g.dense_rows = static_cast<int>(T);
  g.nt = pick_nt_dense(T, (H + 63) / 64);
  g.out = h;
  g.ld_out = H;
  rc = run_gemm(epi_pair, gate, &up, 1, H, D, x, T, D, g, stream);
  if (rc) return rc;
  GemmArgs d = base_args(down, nullptr);
  d.dense_rows = static_cast<int>(T);
  d.nt = pick_nt_dense(T, (D + 127) / 128);
  d.out = out;
  d.ld_out = D;
  if (splits > 1) {
    // Few output tiles: split K over more SMs into fp32 partials, then sum
    // them in order into the output.
    d.out = part;
    d.k_splits = splits;
    d.split_stride = T * D;
    rc = run_gemm(EPI_PLAIN_F32, down, nullptr, 1, D, H, h, T, H, d, stream);
    if (rc) return rc;
    return launch_reduce_splits(part, d.k_splits, T * D, T * D, out, out_dtype == KW8_DT_BF16, stream);
  }
  return run_gemm(epi_out, down, nullptr, 1, D, H, h, T, H, d, stream);
}

int kw8_moe_route(const void* x, int64_t T, int64_t D, int64_t E, int32_t k, kw8_weight router,
                  float* logits_out, int32_t* idx_out, void* w_out, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(x && logits_out && idx_out && w_out, KW8_ERR_INVALID_ARG, "null pointer");
  int rc = check_weight(router, "router");
  if (rc) return rc;
  if (T == 0) return KW8_OK;
  return kw8::route(x, T, D, E, k, router, logits_out, idx_out, w_out, stream);
}

int kw8_moe_topk(const float* logits, int64_t T, int64_t E, int32_t k, int32_t* idx_out,
                 void* w_out, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(logits && idx_out && w_out, KW8_ERR_INVALID_ARG, "null pointer");
  return launch_topk(logits, T, E, k, idx_out, w_out, stream);
}

int kw8_moe_permute(const int32_t* idx, int64_t T, int32_t k, int64_t E, int64_t capacity,
                    int32_t* sorted_token, int32_t* inv_pos, int32_t* group_sizes,
                    int32_t* group_offsets, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(idx && sorted_token && inv_pos && group_sizes && group_offsets, KW8_ERR_INVALID_ARG,
              "null pointer");
  return launch_permute(idx, T, k, E, capacity, sorted_token, inv_pos, group_sizes, group_offsets,
                        stream);
}

size_t kw8_moe_permute_workspace_size(int64_t E) {
  return static_cast<size_t>(permute_hist_ints(E > 0 ? E : 0)) * sizeof(int32_t);
}

int kw8_moe_permute_ws(const int32_t* idx, int64_t T, int32_t k, int64_t E, int64_t capacity,
                       int32_t* sorted_token, int32_t* inv_pos, int32_t* group_sizes,
                       int32_t* group_offsets, void* workspace, size_t workspace_bytes,
                       kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(idx && sorted_token && inv_pos && group_sizes && group_offsets, KW8_ERR_INVALID_ARG,
              "null pointer");
  KW8_REQUIRE(E >= 1, KW8_ERR_INVALID_ARG, "E=%lld invalid", (long long)E);
  KW8_REQUIRE(workspace != nullptr && workspace_bytes >= kw8_moe_permute_workspace_size(E) &&
                  (reinterpret_cast<uintptr_t>(workspace) & 3) == 0,
              KW8_ERR_WORKSPACE, "permute workspace too small (%zu < %zu)", workspace_bytes,
              kw8_moe_permute_workspace_size(E));
  return launch_permute_multi(idx, T, k, E, capacity, static_cast<int32_t*>(workspace), sorted_token,
                              inv_pos, group_sizes, group_offsets, stream, nullptr, nullptr);
}

size_t kw8_moe_expert_ffn_workspace_size(int64_t rows, int64_t D, int64_t I, int64_t E) {
  (void)D;
  Carver c(nullptr, SIZE_MAX);
  carve_expert(c, rows, I, E);
  return c.off;
}

int kw8_moe_expert_ffn(const void* xs, int64_t rows, int64_t D, int64_t I, int64_t E,
                       const int32_t* group_offsets, kw8_weight gate, kw8_weight up,
                       kw8_weight down, void* ys, void* workspace, size_t workspace_bytes,
                       kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(xs && ys && group_offsets, KW8_ERR_INVALID_ARG, "null pointer");
  KW8_REQUIRE(rows >= 0 && D > 0 && I > 0 && E > 0, KW8_ERR_INVALID_ARG, "bad shape");
  int rc = check_weight(gate, "gate");
  if (!rc) rc = check_weight(up, "up");
  if (!rc) rc = check_weight(down, "down");
  if (rc) return rc;
  if (rows == 0) return KW8_OK;
  Carver c(workspace, workspace_bytes);
  ExpertBuffers b = carve_expert(c, rows, I, E);
  KW8_REQUIRE(workspace != nullptr && c.ok, KW8_ERR_WORKSPACE, "expert FFN workspace too small");
  return expert_ffn(use_stream(rows_hint(rows, E)), xs, nullptr, rows, D, I, E, group_offsets, gate,
                    up, down, ys, b, stream);
}

int kw8_moe_combine(const void* ys, const int32_t* inv_pos, const void* w, int64_t T, int32_t k,
                    int64_t D, void* out, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(ys && inv_pos && w && out, KW8_ERR_INVALID_ARG, "null pointer");
  return launch_combine(ys, inv_pos, w, T, k, D, out, stream);
}

size_t kw8_moe_ffn_workspace_size(int64_t T, int64_t D, int64_t I, int64_t E, int32_t k) {
  Carver c(nullptr, SIZE_MAX);
  carve_moe(c, T, D, I, E, k);
  return c.off;
}

int kw8_moe_ffn(const void* x, int64_t T, int64_t D, int64_t I, int64_t E, int32_t k,
                int64_t capacity, kw8_weight router, kw8_weight gate, kw8_weight up,
                kw8_weight down, void* out, void* workspace, size_t workspace_bytes,
                kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(x && out, KW8_ERR_INVALID_ARG, "null x/out");
  int rc = check_moe_args(T, D, I, E, k, router, gate, up, down);
  if (rc || T == 0) return rc;
  Carver c(workspace, workspace_bytes);
  MoeBuffers b = carve_moe(c, T, D, I, E, k);
  KW8_REQUIRE(workspace != nullptr && c.ok, KW8_ERR_WORKSPACE,
              "MoE workspace too small (%zu < %zu)", workspace_bytes, c.off);
  rc = moe_layer_acc(x, T, D, I, E, k, capacity, router, gate, up, down, b, stream);
  if (rc) return rc;
  return launch_f32_to_bf16(b.acc, T * D, out, stream);
}

size_t kw8_moe_block_workspace_size(int64_t T, int64_t D, int64_t I, int64_t E, int32_t k) {
  Carver c(nullptr, SIZE_MAX);
  carve_moe(c, T, D, I, E, k);
  c.take<__nv_bfloat16>(T * D);
  return c.off;
}

int kw8_moe_block(const void* h, int64_t T, int64_t D, int64_t I, int64_t E, int32_t k,
                  int64_t capacity, kw8_weight router, kw8_weight gate, kw8_weight up,
                  kw8_weight down, const kw8_block_norms* norms, void* out, void* workspace,
                  size_t workspace_bytes, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(h && out && h != out, KW8_ERR_INVALID_ARG, "null or aliased h/out");
  int rc = check_moe_args(T, D, I, E, k, router, gate, up, down);
  if (!rc) rc = check_norms(norms, D);
  if (rc || T == 0) return rc;
  Carver c(workspace, workspace_bytes);
  MoeBuffers b = carve_moe(c, T, D, I, E, k);
  __nv_bfloat16* xn = c.take<__nv_bfloat16>(T * D);
  KW8_REQUIRE(workspace != nullptr && c.ok, KW8_ERR_WORKSPACE,
              "MoE block workspace too small (%zu < %zu)", workspace_bytes, c.off);
  rc = launch_rms_norm(h, T, D, norms->pre_scale, norms->scale_dtype, norms->kind, norms->eps, xn, stream);
  if (!rc) rc = moe_layer_acc(xn, T, D, I, E, k, capacity, router, gate, up, down, b, stream);
  if (rc) return rc;
  return launch_block_finish(b.acc, 1, 0, T, D, norms->post_scale, norms->scale_dtype, norms->kind, norms->eps, h,
                             out, stream);
}

size_t kw8_linear_workspace_size(int64_t T, int64_t K, int64_t N) {
  Carver c(nullptr, SIZE_MAX);
  carve_linear(c, T, K, N);
  return c.off;
}

int kw8_linear(const void* x, const int32_t* rows, int64_t T, int64_t K, int64_t N, kw8_weight w,
               int32_t out_dtype, void* out, void* workspace, size_t workspace_bytes,
               kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE((x && out) || T == 0, KW8_ERR_INVALID_ARG, "null x/out");
  KW8_REQUIRE(T >= 0 && K > 0 && N > 0, KW8_ERR_INVALID_ARG, "bad shape (T=%lld K=%lld N=%lld)",
              (long long)T, (long long)K, (long long)N);
  KW8_REQUIRE(out_dtype == KW8_DT_BF16 || out_dtype == KW8_DT_F32, KW8_ERR_INVALID_ARG, "bad out dtype");
  int rc = check_weight(w, "weight");
  if (rc || T == 0) return rc;
  KW8_REQUIRE(T < (1ll << 31) && N < (1ll << 31), KW8_ERR_UNSUPPORTED, "shape out of range");
  Carver c(workspace, workspace_bytes);
  LinearBuffers b = carve_linear(c, T, K, N);
  KW8_REQUIRE(workspace != nullptr && c.ok, KW8_ERR_WORKSPACE, "linear workspace too small (%zu < %zu)",
              workspace_bytes, c.off);
  return linear(x, rows, T, K, N, w, out_dtype == KW8_DT_F32, out, b, stream);
}

int kw8_embed_gather(const int32_t* tokens, int64_t n, kw8_weight table, int64_t V, int64_t D,
                     int32_t out_dtype, void* out, kw8_stream_t stream) {
  KW8_API_BEGIN
  int rc = check_weight(table, "table");
  if (rc) return rc;
  KW8_REQUIRE(table.layout == KW8_LAYOUT_KMAJOR, KW8_ERR_UNSUPPORTED, "embedding tables are gathered K-major");
  return launch_embed_gather(tokens, n, table, V, D, out_dtype, out, stream);
}

int kw8_rms_norm(const void* x, int64_t T, int64_t D, const void* scale, int32_t scale_dtype,
                 int32_t kind, float eps, void* out, kw8_stream_t stream) {
  KW8_API_BEGIN
  return launch_rms_norm(x, T, D, scale, scale_dtype, kind, eps, out, stream);
}

size_t kw8_dense_block_workspace_size(int64_t T, int64_t D, int64_t H) {
  Carver c(nullptr, SIZE_MAX);
  c.take<__nv_bfloat16>(T * D);
  c.take<__nv_bfloat16>(T * H);
  c.take<float>(std::max<int64_t>(dense_down_part_floats(T, D, H), T * D));
  return c.off;
}

int kw8_dense_block(const void* h, int64_t T, int64_t D, int64_t H, kw8_weight gate, kw8_weight up,
                    kw8_weight down, int32_t act, const kw8_block_norms* norms, void* out,
                    void* workspace, size_t workspace_bytes, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(h && out && h != out, KW8_ERR_INVALID_ARG, "null or aliased h/out");
  KW8_REQUIRE(T >= 0 && D > 0 && H > 0, KW8_ERR_INVALID_ARG, "bad shape");
  KW8_REQUIRE(act == KW8_ACT_GELU_TANH || act == KW8_ACT_SILU, KW8_ERR_INVALID_ARG, "bad act");
  int rc = check_weight(gate, "gate");
  if (!rc) rc = check_weight(up, "up");
  if (!rc) rc = check_weight(down, "down");
  if (!rc) rc = check_norms(norms, D);
  if (rc || T == 0) return rc;
  KW8_REQUIRE(T < (1ll << 31), KW8_ERR_UNSUPPORTED, "too many tokens");
  Carver c(workspace, workspace_bytes);
  __nv_bfloat16* xn = c.take<__nv_bfloat16>(T * D);
  __nv_bfloat16* hid = c.take<__nv_bfloat16>(T * H);
  float* part = c.take<float>(std::max<int64_t>(dense_down_part_floats(T, D, H), T * D));
  KW8_REQUIRE(workspace != nullptr && c.ok, KW8_ERR_WORKSPACE, "dense block workspace too small (%zu < %zu)",
              workspace_bytes, c.off);
  const int splits = dense_down_splits(T, D, H);
  rc = launch_rms_norm(h, T, D, norms->pre_scale, norms->scale_dtype, norms->kind, norms->eps, xn, stream);
  if (!rc) rc = dense_gate_up(xn, T, D, H, gate, up, act, hid, stream);
  if (!rc) rc = dense_f32_parts(hid, T, H, D, down, splits, part, stream);
  if (rc) return rc;
  // One pass per row: the split sums, bf16, the post-FFN norm, the residual.
  return launch_block_finish(part, splits, T * D, T, D, norms->post_scale, norms->scale_dtype, norms->kind,
                             norms->eps, h, out, stream);
}

}  // extern "C"
