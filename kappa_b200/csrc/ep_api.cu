// C ABI of the expert-parallel row movement and its CUDA-IPC buffers.
#include <cstring>

#include "ep.cuh"

namespace kw8 {
namespace {

// Workspace of kw8_moe_ffn_ep: routing of up to max_tokens tokens, the
// local experts' offsets, and the expert FFN over the receive buffer's
// world * max_tokens * k rows (tile table, h, outputs).
struct EpBuffers {
  float* logits;
  int32_t* idx;
  __nv_bfloat16* w;
  int32_t* sorted_token;
  int32_t* inv_pos;
  int32_t* group_sizes;
  int32_t* group_offsets;
  int32_t* perm_hist;
  int32_t* loc_off;
  ExpertBuffers eb;
  __nv_bfloat16* ys_loc;  // expert outputs (or, deduplicated path, the gathered rows)
  // Deduplicated path only.
  float* sorted_w;
  int32_t* tok_slot;  // [max_tokens][world]
  int32_t* u_cnt;     // [world]
  float* part;        // [world * max_tokens][D] fp32 partial sums
};

EpBuffers carve_ep(Carver& c, int64_t max_tokens, int64_t D, int64_t I, int64_t E, int k, int world) {
  EpBuffers b;
  const int64_t m = max_tokens * k;
  const int64_t e_loc = std::max<int64_t>(1, E / std::max(world, 1));
  const int64_t recv_rows = static_cast<int64_t>(world) * m;
  b.logits = c.take<float>(max_tokens * E);
  b.idx = c.take<int32_t>(m);
  b.w = c.take<__nv_bfloat16>(m);
  b.sorted_token = c.take<int32_t>(m);
  b.inv_pos = c.take<int32_t>(m);
  b.group_sizes = c.take<int32_t>(E);
  b.group_offsets = c.take<int32_t>(E + 1);
  b.perm_hist = c.take<int32_t>(permute_hist_ints(E));
  b.loc_off = c.take<int32_t>(e_loc + 1);
  b.eb = carve_expert(c, recv_rows, I, e_loc);
  b.ys_loc = c.take<__nv_bfloat16>(recv_rows * D);
  b.sorted_w = c.take<float>(m);
  b.tok_slot = c.take<int32_t>(max_tokens * world);
  b.u_cnt = c.take<int32_t>(kEpMaxRanks);
  b.part = c.take<float>(static_cast<int64_t>(world) * max_tokens * D);
  return b;
}

// The members every group call needs: rank, world, flags and (for the
// one-shot sums) the exchange buffer.
int check_group(const kw8_ep_peers* p) {
  KW8_REQUIRE(p != nullptr, KW8_ERR_INVALID_ARG, "null peers");
  KW8_REQUIRE(p->world >= 1 && p->world <= kEpMaxRanks && p->rank >= 0 && p->rank < p->world,
              KW8_ERR_INVALID_ARG, "bad rank %d of %d", p->rank, p->world);
  KW8_REQUIRE(p->flags && p->own_flags && p->red && p->own_red && p->red_rows >= 0, KW8_ERR_INVALID_ARG,
              "incomplete peers (flags and the exchange buffer are required)");
  return KW8_OK;
}

// Phase timing of kw8_moe_ffn_ep (option 4): CUDA events recorded on the
// call's stream at the phase boundaries of the last call on each device.
constexpr int kEpPhases = 9;
cudaEvent_t g_ep_events[64][kEpPhases + 1] = {};
bool g_ep_recorded[64] = {};

struct PhaseClock {
  int dev = -1;
  cudaStream_t stream;
  explicit PhaseClock(cudaStream_t s) : stream(s) {
    if (!g_opt_ep_timing.load()) return;
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 64) return;
    for (int i = 0; i <= kEpPhases; ++i)
      if (g_ep_events[d][i] == nullptr && cudaEventCreate(&g_ep_events[d][i]) != cudaSuccess) return;
    dev = d;
    g_ep_recorded[d] = false;
    mark(0);
  }
  void mark(int i) {
    if (dev >= 0) cudaEventRecord(g_ep_events[dev][i], stream);
  }
  void done() {
    if (dev >= 0) {
      mark(kEpPhases);
      g_ep_recorded[dev] = true;
    }
  }
};

int check_peers(const kw8_ep_peers* p) {
  KW8_REQUIRE(p != nullptr, KW8_ERR_INVALID_ARG, "null peers");
  KW8_REQUIRE(p->world >= 1 && p->world <= kEpMaxRanks && p->rank >= 0 && p->rank < p->world,
              KW8_ERR_INVALID_ARG, "bad rank %d of %d", p->rank, p->world);
  KW8_REQUIRE(p->recv && p->out && p->counts && p->flags && p->own_recv && p->own_out &&
                  p->own_counts && p->own_flags && p->max_tokens >= 0,
              KW8_ERR_INVALID_ARG, "incomplete peers");
  return KW8_OK;
}

}  // namespace
}  // namespace kw8

using namespace kw8;

extern "C" {

size_t kw8_ipc_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

int kw8_ipc_alloc(size_t bytes, void** ptr_out, void* handle_out) {
  KW8_API_BEGIN
  KW8_REQUIRE(ptr_out && handle_out && bytes > 0, KW8_ERR_INVALID_ARG, "bad ipc_alloc args");
  void* p = nullptr;
  KW8_CUDA_TRY(cudaMalloc(&p, bytes));
  // Zeroed before any peer can map it (the group flags start at zero).
  cudaError_t z = cudaMemset(p, 0, bytes);
  if (z == cudaSuccess) z = cudaDeviceSynchronize();
  if (z != cudaSuccess) {
    cudaFree(p);
    return fail(KW8_ERR_CUDA, "zeroing the ipc buffer: %s", cudaGetErrorString(z));
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(KW8_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *ptr_out = p;
  return KW8_OK;
}

int kw8_ipc_free(void* ptr) {
  KW8_API_BEGIN
  if (ptr) KW8_CUDA_TRY(cudaFree(ptr));
  return KW8_OK;
}

int kw8_ipc_open(const void* handle, void** ptr_out) {
  KW8_API_BEGIN
  KW8_REQUIRE(handle && ptr_out, KW8_ERR_INVALID_ARG, "bad ipc_open args");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  KW8_CUDA_TRY(cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess));
  return KW8_OK;
}

int kw8_ipc_close(void* ptr) {
  KW8_API_BEGIN
  if (ptr) KW8_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return KW8_OK;
}

int kw8_ep_dispatch(const void* x, int64_t max_rows, int64_t D, const int32_t* sorted_token,
                    const int32_t* group_offsets, const int32_t* counts, int32_t world, int32_t rank,
                    int64_t E, const uint64_t* peer_recv, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(x && sorted_token && group_offsets && counts && peer_recv, KW8_ERR_INVALID_ARG,
              "null pointer");
  return launch_ep_dispatch(x, max_rows, D, sorted_token, group_offsets, counts, world, rank, E,
                            peer_recv, static_cast<cudaStream_t>(stream));
}

int kw8_ep_return(const void* ys, int64_t max_rows, int64_t D, const int32_t* counts, int32_t world,
                  int32_t rank, int64_t E, const uint64_t* peer_out, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(ys && counts && peer_out, KW8_ERR_INVALID_ARG, "null pointer");
  return launch_ep_return(ys, max_rows, D, counts, world, rank, E, peer_out,
                          static_cast<cudaStream_t>(stream));
}

int kw8_ep_local_offsets(const int32_t* counts, int32_t world, int32_t rank, int64_t E,
                         int32_t* local_offsets, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(counts && local_offsets, KW8_ERR_INVALID_ARG, "null pointer");
  return launch_ep_local_offsets(counts, world, rank, E, local_offsets,
                                 static_cast<cudaStream_t>(stream));
}

size_t kw8_moe_ffn_ep_workspace_size(int64_t max_tokens, int64_t D, int64_t I, int64_t E,
                                     int32_t k, int32_t world) {
  Carver c(nullptr, SIZE_MAX);
  carve_ep(c, max_tokens, D, I, E, k, world);
  return c.off;
}

int kw8_moe_ffn_ep(const void* x, int64_t T, int64_t D, int64_t I, int64_t E, int32_t k,
                   int64_t capacity, kw8_weight router, kw8_weight gate_local,
                   kw8_weight up_local, kw8_weight down_local, void* out,
                   const kw8_ep_peers* peers, uint32_t epoch, void* workspace,
                   size_t workspace_bytes, kw8_stream_t stream_in) {
  KW8_API_BEGIN
  int rc = check_peers(peers);
  if (rc) return rc;
  const int world = peers->world, rank = peers->rank;
  KW8_REQUIRE((x && out) || T == 0, KW8_ERR_INVALID_ARG, "null x/out");
  KW8_REQUIRE(T >= 0 && T <= peers->max_tokens && D > 0 && I > 0 && k >= 1 && k <= E,
              KW8_ERR_INVALID_ARG, "bad shape (T=%lld of at most %lld, D=%lld, I=%lld, k=%d)",
              (long long)T, (long long)peers->max_tokens, (long long)D, (long long)I, k);
  rc = check_ep(D, world, rank, E);
  if (!rc) rc = check_weight(router, "router");
  if (!rc) rc = check_weight(gate_local, "gate");
  if (!rc) rc = check_weight(up_local, "up");
  if (!rc) rc = check_weight(down_local, "down");
  if (rc) return rc;
  Carver c(workspace, workspace_bytes);
  EpBuffers b = carve_ep(c, peers->max_tokens, D, I, E, k, world);
  KW8_REQUIRE(workspace != nullptr && c.ok, KW8_ERR_WORKSPACE, "EP workspace too small (%zu < %zu)",
              workspace_bytes, c.off);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_in);
  const int64_t e_loc = E / world;
  const int64_t recv_rows = static_cast<int64_t>(world) * peers->max_tokens * k;
  PhaseClock clock(stream);
  // Route and permute this rank's tokens (a rank without tokens still takes
  // part: its counts are zero).
  if (T > 0) {
    rc = kw8::route(x, T, D, E, k, router, b.logits, b.idx, b.w, stream);
    if (rc) return rc;
  }
  const bool dedup = peers->rows != nullptr;
  rc = launch_permute_multi(b.idx, T, k, E, capacity, b.perm_hist, b.sorted_token, b.inv_pos,
                            b.group_sizes, b.group_offsets, stream, dedup ? b.w : nullptr,
                            dedup ? b.sorted_w : nullptr);
  if (rc) return rc;
  clock.mark(1);
  if (dedup) {
    // Each token once per owning rank (ep_dedup.cu).
    KW8_REQUIRE(peers->meta && peers->ret && peers->own_rows && peers->own_meta && peers->own_ret &&
                    D % 8 == 0 && peers->ret_format >= KW8_RET_BF16 && peers->ret_format <= KW8_RET_F16_SCALED,
                KW8_ERR_INVALID_ARG, "incomplete peers for the deduplicated step");
    const int64_t pair_cap = recv_rows;
    rc = launch_ep_slots(b.idx, b.inv_pos, T, k, E, world, b.tok_slot, b.u_cnt, stream);
    if (rc) return rc;
    rc = launch_ep_counts2(b.group_sizes, b.u_cnt, E, peers->counts, peers->flags, peers->own_flags, world,
                           rank, epoch, stream);
    if (rc) return rc;
    clock.mark(2);
    const int32_t* cnt = peers->own_counts + static_cast<int64_t>(epoch & 1u) * world * (E + world);
    rc = launch_ep_dispatch2(x, T, k, D, b.sorted_token, b.group_offsets, b.sorted_w, b.tok_slot, cnt, world,
                             rank, E, pair_cap, peers->rows, peers->meta, stream);
    if (rc) return rc;
    clock.mark(3);
    rc = launch_ep_barrier(peers->flags, peers->own_flags, world, rank, 1, epoch, true, stream);
    if (rc) return rc;
    clock.mark(4);
    rc = launch_ep_local_offsets(cnt, world, rank, E, b.loc_off, stream, E + world);
    if (rc) return rc;
    const int32_t* meta_u = static_cast<const int32_t*>(peers->own_meta);
    const float* meta_w = reinterpret_cast<const float*>(meta_u + pair_cap);
    rc = launch_ep_gather2(peers->own_rows, meta_u, b.loc_off, e_loc, cnt, world, rank, E, D, recv_rows,
                           b.ys_loc, b.part, stream);
    if (rc) return rc;
    clock.mark(5);
    // The down projection adds w * y of every pair into its token's fp32
    // partial row (rows indexed by the pair records).
    rc = expert_ffn(use_stream(rows_hint(recv_rows, e_loc)), b.ys_loc, nullptr, recv_rows, D, I, e_loc,
                    b.loc_off, gate_local, up_local, down_local, b.part, b.eb, stream, meta_u, meta_w);
    if (rc) return rc;
    clock.mark(6);
    rc = launch_ep_return2(b.part, D, cnt, world, rank, E, peers->max_tokens, peers->ret, peers->ret_format,
                           stream);
    if (rc) return rc;
    clock.mark(7);
    rc = launch_ep_barrier(peers->flags, peers->own_flags, world, rank, 2, epoch, true, stream);
    if (rc) return rc;
    clock.mark(8);
    rc = launch_ep_final2(peers->own_ret, b.tok_slot, T, world, peers->max_tokens, D, peers->ret_format, out,
                          stream);
    if (!rc) clock.done();
    return rc;
  }
  // Counts to every peer (phase 0), rows to their expert owners (phase 1).
  rc = launch_ep_counts(b.group_sizes, E, peers->counts, peers->flags, peers->own_flags, world, rank,
                        epoch, stream);
  if (rc) return rc;
  const int32_t* counts = peers->own_counts + static_cast<int64_t>(epoch & 1u) * world * E;
  rc = launch_ep_dispatch(x, T * k, D, b.sorted_token, b.group_offsets, counts, world, rank, E,
                          peers->recv, stream);
  if (rc) return rc;
  rc = launch_ep_barrier(peers->flags, peers->own_flags, world, rank, 1, epoch, true, stream);
  if (rc) return rc;
  // The local experts over every rank's rows, outputs back to their
  // sources (phase 2), then the weighted combine of this rank's tokens.
  // (Stores of the output rows to the sources from the down GEMM's
  // epilogue, 64 bytes per row and tile over NVLink, were measured slower:
  // 0.91 vs 0.78 ms per 2-GPU step.)
  rc = launch_ep_local_offsets(counts, world, rank, E, b.loc_off, stream);
  if (rc) return rc;
  rc = expert_ffn(use_stream(rows_hint(recv_rows, e_loc)), peers->own_recv, nullptr, recv_rows, D, I,
                  e_loc, b.loc_off, gate_local, up_local, down_local, b.ys_loc, b.eb, stream);
  if (rc) return rc;
  rc = launch_ep_return(b.ys_loc, recv_rows, D, counts, world, rank, E, peers->out, stream);
  if (rc) return rc;
  rc = launch_ep_barrier(peers->flags, peers->own_flags, world, rank, 2, epoch, true, stream);
  if (rc) return rc;
  return launch_combine(peers->own_out, b.inv_pos, b.w, T, k, D, out, stream);
}

size_t kw8_moe_ffn_ep_decode_workspace_size(int64_t T, int64_t D, int64_t I, int64_t E, int32_t k) {
  Carver c(nullptr, SIZE_MAX);
  carve_moe(c, T, D, I, E, k);
  return c.off;
}

int kw8_moe_ffn_ep_decode(const void* x, int64_t T, int64_t D, int64_t I, int64_t E, int32_t k,
                          int64_t capacity, kw8_weight router, kw8_weight gate_local,
                          kw8_weight up_local, kw8_weight down_local, void* out,
                          const kw8_ep_peers* peers, uint32_t epoch, void* workspace,
                          size_t workspace_bytes, kw8_stream_t stream_in) {
  KW8_API_BEGIN
  int rc = check_group(peers);
  if (rc) return rc;
  const int world = peers->world, rank = peers->rank;
  KW8_REQUIRE((x && out) || T == 0, KW8_ERR_INVALID_ARG, "null x/out");
  rc = check_ep(D, world, rank, E);
  if (!rc) rc = check_moe_args(T, D, I, E, k, router, gate_local, up_local, down_local);
  if (rc) return rc;
  KW8_REQUIRE(T <= peers->red_rows, KW8_ERR_UNSUPPORTED, "T=%lld exceeds the group's exchange rows (%lld)",
              (long long)T, (long long)peers->red_rows);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_in);
  Carver c(workspace, workspace_bytes);
  MoeBuffers b = carve_moe(c, T, D, I, E, k);
  KW8_REQUIRE(workspace != nullptr && c.ok, KW8_ERR_WORKSPACE, "EP decode workspace too small (%zu < %zu)",
              workspace_bytes, c.off);
  const int64_t e_loc = E / world;
  const int64_t m = T * k;
  if (T > 0) {
    // Every rank routes every token: the same logits, top-k and permutation.
    float* part = router_part_floats(T, D, E) > 0 ? b.router_part : nullptr;
    if (route_tail_small_ok(T, E, k)) {
      rc = router_logits(x, T, D, E, router, b.logits, stream, part);
      if (!rc)
        rc = launch_route_tail_small(b.logits, T, E, k, capacity, b.idx, b.w, b.sorted_token, b.inv_pos,
                                     b.group_sizes, b.group_offsets, b.sorted_w, b.active, b.acc, D, stream);
    } else {
      rc = kw8::route(x, T, D, E, k, router, b.logits, b.idx, b.w, stream, part, b.acc, D);
      if (!rc)
        rc = launch_permute_multi(b.idx, T, k, E, capacity, b.perm_hist, b.sorted_token, b.inv_pos,
                                  b.group_sizes, b.group_offsets, stream, b.w, b.sorted_w, b.active);
    }
    if (rc) return rc;
    // This rank's experts: their rows are a contiguous range of the sorted
    // order (offsets e_loc * rank .. e_loc * (rank + 1)); the fused combine
    // adds their weighted outputs into the fp32 partial b.acc.
    const bool streamed = use_stream(rows_hint(m, E));
    if (!streamed) {
      rc = launch_gather(x, b.sorted_token, b.group_offsets + E, m, D, b.xs, stream);
      if (rc) return rc;
    }
    ExpertBuffers eb{b.tiles, b.num_tiles, b.h};
    const int64_t m_loc = std::max<int64_t>(1, m * e_loc / E);  // expected local rows (tile choice)
    rc = expert_ffn(streamed, streamed ? x : b.xs, streamed ? b.sorted_token : nullptr, m, D, I, e_loc,
                    b.group_offsets + rank * e_loc, gate_local, up_local, down_local, b.acc, eb, stream,
                    b.sorted_token, b.sorted_w, nullptr, m_loc);
    if (rc) return rc;
  }
  return launch_ep_allreduce(b.acc, 1, 0, T, D, peers->red, peers->own_red, peers->red_rows, peers->flags,
                             peers->own_flags, world, rank, epoch, out, stream);
}

size_t kw8_dense_ffn_tp_workspace_size(int64_t T, int64_t D, int64_t H_local) {
  Carver c(nullptr, SIZE_MAX);
  c.take<__nv_bfloat16>(T * H_local);
  c.take<float>(std::max<int64_t>(dense_down_part_floats(T, D, H_local), T * D));
  return c.off;
}

int kw8_dense_ffn_tp(const void* x, int64_t T, int64_t D, int64_t H_local, kw8_weight gate,
                     kw8_weight up, kw8_weight down, int32_t act, void* out,
                     const kw8_ep_peers* peers, uint32_t epoch, void* workspace,
                     size_t workspace_bytes, kw8_stream_t stream_in) {
  KW8_API_BEGIN
  int rc = check_group(peers);
  if (rc) return rc;
  KW8_REQUIRE((x && out) || T == 0, KW8_ERR_INVALID_ARG, "null x/out");
  KW8_REQUIRE(T >= 0 && D > 0 && D % 8 == 0 && H_local > 0, KW8_ERR_INVALID_ARG, "bad shape");
  KW8_REQUIRE(act == KW8_ACT_GELU_TANH || act == KW8_ACT_SILU, KW8_ERR_INVALID_ARG, "bad act");
  rc = check_weight(gate, "gate");
  if (!rc) rc = check_weight(up, "up");
  if (!rc) rc = check_weight(down, "down");
  if (rc) return rc;
  KW8_REQUIRE(T <= peers->red_rows, KW8_ERR_UNSUPPORTED, "T=%lld exceeds the group's exchange rows (%lld)",
              (long long)T, (long long)peers->red_rows);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_in);
  Carver c(workspace, workspace_bytes);
  __nv_bfloat16* hid = c.take<__nv_bfloat16>(T * H_local);
  float* part = c.take<float>(std::max<int64_t>(dense_down_part_floats(T, D, H_local), T * D));
  KW8_REQUIRE(workspace != nullptr && c.ok, KW8_ERR_WORKSPACE, "TP workspace too small (%zu < %zu)",
              workspace_bytes, c.off);
  const int splits = T > 0 ? dense_down_splits(T, D, H_local) : 1;
  if (T > 0) {
    rc = dense_gate_up(x, T, D, H_local, gate, up, act, hid, stream);
    if (!rc) rc = dense_f32_parts(hid, T, H_local, D, down, splits, part, stream);
    if (rc) return rc;
  }
  // The K-split slices of this rank's partial are summed while they are pushed.
  return launch_ep_allreduce(part, splits, T * D, T, D, peers->red, peers->own_red, peers->red_rows,
                             peers->flags, peers->own_flags, peers->world, peers->rank, epoch, out, stream);
}

int kw8_ep_phase_times(float* ms_out, int32_t n) {
  KW8_API_BEGIN
  int dev = 0;
  KW8_CUDA_TRY(cudaGetDevice(&dev));
  KW8_REQUIRE(ms_out && n >= 1 && dev >= 0 && dev < 64, KW8_ERR_INVALID_ARG, "bad arguments");
  KW8_REQUIRE(g_ep_recorded[dev], KW8_ERR_INVALID_ARG,
              "no timed kw8_moe_ffn_ep call on this device (set option 4 and take the deduplicated step)");
  KW8_CUDA_TRY(cudaEventSynchronize(g_ep_events[dev][kEpPhases]));
  for (int i = 0; i < n && i < kEpPhases; ++i)
    KW8_CUDA_TRY(cudaEventElapsedTime(&ms_out[i], g_ep_events[dev][i], g_ep_events[dev][i + 1]));
  return KW8_OK;
}

int kw8_ep_barrier(const kw8_ep_peers* peers, int32_t phase, uint32_t epoch, int32_t signal,
                   kw8_stream_t stream) {
  KW8_API_BEGIN
  int rc = check_peers(peers);
  if (rc) return rc;
  return launch_ep_barrier(peers->flags, peers->own_flags, peers->world, peers->rank, phase, epoch,
                           signal != 0, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
