// MoE routing kernels: top-k + softmax, stable expert permutation,
// tile-table construction, row gather and the weighted combine.
#include "moe.cuh"

namespace kw8 {

namespace {

constexpr int kBlock = 1024;
constexpr int kPermBatch = 16;  // 32-entry steps per lane fetched at once
constexpr int kPermThreads = 256;

// Block-wide exclusive scan of one int per thread (blockDim.x a multiple of
// 32).  Returns the exclusive prefix; *total receives the block sum.
__device__ int block_exclusive_scan(int v, int* total) {
  __shared__ int warp_sums[32];
  __shared__ int total_sh;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int s = lane < static_cast<int>(blockDim.x >> 5) ? warp_sums[lane] : 0;
    int si = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, si, o);
      if (lane >= o) si += n;
    }
    warp_sums[lane] = si - s;
    if (lane == 31) total_sh = si;
  }
  __syncthreads();
  const int r = warp_sums[warp] + incl - v;
  *total = total_sh;
  __syncthreads();
  return r;
}

// ------------------------------------------------------------- top-k ----
// One warp per token.  Lane l holds logits l, l+32, ... (E <= 32*kMaxPerLane).
// Round j picks the largest remaining logit, ties to the lower index, which
// is jax.lax.top_k's order; lane j keeps round j's winner.  The softmax over
// the k winners is fp32 exp(v - max) / sum, rounded to bf16.
constexpr int kMaxPerLane = 8;

// Top-k + softmax of one logit row by one warp: lane j < k receives the
// j-th winner and its bf16 weight.
__device__ __forceinline__ void topk_row(const float* __restrict__ row, int E, int k, int lane,
                                         int* my_idx, __nv_bfloat16* my_w) {
  float v[kMaxPerLane];
  bool taken[kMaxPerLane];
#pragma unroll
  for (int i = 0; i < kMaxPerLane; ++i) {
    const int e = lane + 32 * i;
    v[i] = (e < E) ? row[e] : 0.f;
    taken[i] = !(e < E);
  }
  float my_v = -INFINITY;
  int my_i = -1;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int e = lane + 32 * i;
      if (!taken[i] && (v[i] > bv || (v[i] == bv && e < bi))) {
        bv = v[i];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i)
      if (lane + 32 * i == bi) taken[i] = true;
    if (lane == j) {
      my_v = bv;
      my_i = bi;
    }
  }
  const float m = __shfl_sync(0xffffffffu, my_v, 0);
  const float ex = (lane < k) ? expf(my_v - m) : 0.f;
  float s = ex;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  *my_idx = my_i;
  *my_w = __float2bfloat16_rn(__fdiv_rn(ex, s));
}

__global__ void topk_softmax_kernel(const float* __restrict__ logits, int T, int E, int k,
                                    int32_t* __restrict__ idx_out,
                                    __nv_bfloat16* __restrict__ w_out, float4* __restrict__ zero_rows,
                                    int zero_vec4) {
  const int lane = threadIdx.x & 31;
  const int tok = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (tok >= T) return;
  // Optional: this token's row of a buffer the caller needs zeroed (the
  // fp32 combine buffer the down projection adds into).
  if (zero_rows != nullptr)
    for (int c = lane; c < zero_vec4; c += 32)
      zero_rows[static_cast<int64_t>(tok) * zero_vec4 + c] = make_float4(0.f, 0.f, 0.f, 0.f);
  int my_i;
  __nv_bfloat16 my_w;
  topk_row(logits + static_cast<int64_t>(tok) * E, E, k, lane, &my_i, &my_w);
  if (lane < k) {
    idx_out[static_cast<int64_t>(tok) * k + lane] = my_i;
    w_out[static_cast<int64_t>(tok) * k + lane] = my_w;
  }
}

// ------------------------------------------------ small routing tail ----
// Everything between the router logits and the expert GEMMs for a handful
// of tokens, in one CTA of kTailThreads: top-k + softmax of every token (one
// warp per token, topk_row as above), then the same stable permutation as
// permute_kernel (entries sorted by expert, ties by flat index, at most
// `capacity` rows per expert), the active-expert list, and the zeroing of
// the fp32 combine buffer.  The rank of entry i among its expert's entries
// is the count of equal experts before it, read from shared memory (m <=
// kTailMaxRows entries, so the quadratic count is a few hundred steps).
constexpr int kTailThreads = 256;

__global__ void __launch_bounds__(kTailThreads)
    route_tail_small_kernel(const float* __restrict__ logits, int T, int E, int k, int capacity,
                            int32_t* __restrict__ idx_out, __nv_bfloat16* __restrict__ w_out,
                            int32_t* __restrict__ sorted_token, int32_t* __restrict__ inv_pos,
                            int32_t* __restrict__ group_sizes, int32_t* __restrict__ group_offsets,
                            float* __restrict__ sorted_w, int32_t* __restrict__ active,
                            float4* __restrict__ zero_rows, int zero_vec4) {
  __shared__ int ent_e[kTailMaxRows];    // expert of flat entry i = t * k + j
  __shared__ float ent_w[kTailMaxRows];  // its weight, bf16 value in fp32
  __shared__ int cnt[kTailThreads];      // entries per expert (E <= kTailThreads)
  __shared__ int goff[kTailThreads];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int m = T * k;
  cnt[threadIdx.x] = 0;
  if (zero_rows != nullptr)
    for (int c = threadIdx.x; c < T * zero_vec4; c += kTailThreads)
      zero_rows[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int tok = warp; tok < T; tok += kTailThreads / 32) {
    int my_i;
    __nv_bfloat16 my_w;
    topk_row(logits + static_cast<int64_t>(tok) * E, E, k, lane, &my_i, &my_w);
    if (lane < k) {
      idx_out[tok * k + lane] = my_i;
      w_out[tok * k + lane] = my_w;
      // A row without k ordered logits (NaN, or -inf everywhere) yields no
      // expert: reported like an invalid id in the permutation, and dropped.
      const bool valid = my_i >= 0 && my_i < E;
      if (!valid) report(KW8_ERR_INVALID_ARG);
      ent_e[tok * k + lane] = valid ? my_i : -1;
      ent_w[tok * k + lane] = __bfloat162float(my_w);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < m; i += kTailThreads)
    if (ent_e[i] >= 0) atomicAdd(&cnt[ent_e[i]], 1);
  __syncthreads();
  const int e = threadIdx.x;
  const int kept = e < E ? (capacity >= 0 ? min(cnt[e], capacity) : cnt[e]) : 0;
  int total, n_active;
  const int off = block_exclusive_scan(kept, &total);
  const int apos = block_exclusive_scan(kept > 0 ? 1 : 0, &n_active);
  if (e < E) {
    group_sizes[e] = kept;
    group_offsets[e] = off;
    goff[e] = off;
    if (kept > 0) active[1 + apos] = e;
  }
  if (threadIdx.x == 0) {
    group_offsets[E] = total;
    active[0] = n_active;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < m; i += kTailThreads) {
    const int ei = ent_e[i];
    if (ei < 0) {
      inv_pos[i] = -1;
      continue;
    }
    int rank = 0;
    for (int j = 0; j < i; ++j) rank += (ent_e[j] == ei) ? 1 : 0;
    if (capacity < 0 || rank < capacity) {
      const int p = goff[ei] + rank;
      sorted_token[p] = i / k;
      inv_pos[i] = p;
      sorted_w[p] = ent_w[i];
    } else {
      inv_pos[i] = -1;
    }
  }
}

// ----------------------------------------------------------- permute ----
// Stable counting sort of the T*k expert ids in one CTA of 32 warps.  Warp w
// owns a contiguous chunk of entries and walks it 32 at a time; lanes with
// the same expert find each other with __match_any_sync, so a lane's rank
// among equal experts in the step is the number of lower lanes that match.
// Pass 1 counts per (warp, expert); the counts become per-(warp, expert)
// start slots; pass 2 assigns slots in the same order.  The result is the
// order of a stable argsort by expert id (ties by flat index).
__global__ void __launch_bounds__(kBlock, 1)
    permute_kernel(const int32_t* __restrict__ idx, int m, int k, int E, int capacity,
                   int32_t* __restrict__ sorted_token, int32_t* __restrict__ inv_pos,
                   int32_t* __restrict__ group_sizes, int32_t* __restrict__ group_offsets,
                   const __nv_bfloat16* __restrict__ w, float* __restrict__ sorted_w) {
  extern __shared__ int sm[];
  int* cnt = sm;            // [32][E]
  int* goff = sm + 32 * E;  // [E]
  __shared__ int total_sh;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < 32 * E; i += kBlock) cnt[i] = 0;
  __syncthreads();

  const int chunk = ((m + 31) / 32 + 31) & ~31;
  const int beg = warp * chunk;
  const int end = min(m, beg + chunk);
  // Each lane's ids are fetched kPermBatch steps at a time (independent
  // loads in flight) before the warp walks them.
  for (int b0 = beg; b0 < end; b0 += 32 * kPermBatch) {
    int ev[kPermBatch];
#pragma unroll
    for (int s = 0; s < kPermBatch; ++s) {
      const int i = b0 + s * 32 + lane;
      ev[s] = (i < end) ? idx[i] : -1;
    }
#pragma unroll
    for (int s = 0; s < kPermBatch; ++s) {
      const int i = b0 + s * 32 + lane;
      int e = ev[s];
      if (i < end && (e < 0 || e >= E)) {
        report(KW8_ERR_INVALID_ARG);
        e = -1;
      }
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * E + e] += __popc(peers);
    }
  }
  __syncthreads();

  for (int e0 = 0; e0 < E; e0 += kBlock) {
    const int e = e0 + threadIdx.x;
    int kept = 0;
    if (e < E) {
      int acc = 0;
      for (int w = 0; w < 32; ++w) {
        const int c = cnt[w * E + e];
        cnt[w * E + e] = acc;
        acc += c;
      }
      kept = capacity >= 0 ? min(acc, capacity) : acc;
      group_sizes[e] = kept;
    }
    int tot;
    const int off = block_exclusive_scan(kept, &tot);
    const int carry = (e0 == 0) ? 0 : total_sh;
    if (e < E) {
      goff[e] = carry + off;
      group_offsets[e] = carry + off;
    }
    __syncthreads();
    if (threadIdx.x == 0) total_sh = carry + tot;
    __syncthreads();
  }
  if (threadIdx.x == 0) group_offsets[E] = total_sh;
  __syncthreads();

  for (int b0 = beg; b0 < end; b0 += 32 * kPermBatch) {
    int ev[kPermBatch];
    float wv[kPermBatch];
#pragma unroll
    for (int s = 0; s < kPermBatch; ++s) {
      const int i = b0 + s * 32 + lane;
      ev[s] = (i < end) ? idx[i] : -1;
      wv[s] = (i < end && sorted_w != nullptr) ? __bfloat162float(w[i]) : 0.f;
    }
#pragma unroll
    for (int s = 0; s < kPermBatch; ++s) {
      const int i = b0 + s * 32 + lane;
      int e = ev[s];
      if (e >= E || e < 0) e = -1;
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      if (e >= 0) {
        const int rank = __popc(peers & ((1u << lane) - 1u));
        const int slot = cnt[warp * E + e] + rank;
        if (capacity < 0 || slot < capacity) {
          const int p = goff[e] + slot;
          sorted_token[p] = i / k;
          inv_pos[i] = p;
          if (sorted_w != nullptr) sorted_w[p] = wv[s];
        } else {
          inv_pos[i] = -1;
        }
      } else if (i < end) {
        inv_pos[i] = -1;
      }
      __syncwarp();
      if (e >= 0 && lane == __ffs(peers) - 1) cnt[warp * E + e] += __popc(peers);
      __syncwarp();
    }
  }
}

// ------------------------------------------- multi-block stable permute ----
// The same permutation as permute_kernel, spread over up to kPermMaxBlocks
// blocks of kPermThreads: block b owns the flat range [b*chunk, (b+1)*chunk).
// Pass 1 writes each block's expert histogram; pass 2 gives every block its
// first slot per expert (the counts of all lower blocks), the expert offsets
// (scan of the capacity-clipped totals) and scatters its entries, ranking
// equal experts within a 256-entry round by warp (ballot match) and lane.

// Pass 1: hist[b][e] = entries of block b routed to expert e.
__global__ void __launch_bounds__(kPermThreads)
    permute_hist_kernel(const int32_t* __restrict__ idx, int m, int E, int chunk,
                        int32_t* __restrict__ hist) {
  extern __shared__ int cnt[];  // [E]
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  const int beg = blockIdx.x * chunk;
  const int end = min(m, beg + chunk);
  for (int i = beg + threadIdx.x; i < end; i += blockDim.x) {
    const int e = idx[i];
    if (e >= 0 && e < E)
      atomicAdd(&cnt[e], 1);
    else
      report(KW8_ERR_INVALID_ARG);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[blockIdx.x * E + e] = cnt[e];
}

// Pass 2: offsets and stable scatter (see above).  Shared memory: base[E]
// (this block's first slot per expert), goff[E] (expert offsets), run[E]
// (entries of earlier rounds), wcnt[kPermThreads/32][E] (per-warp counts of
// the current round, zero between rounds).
__global__ void __launch_bounds__(kPermThreads)
    permute_scatter_kernel(const int32_t* __restrict__ idx, int m, int k, int E, int capacity,
                           int chunk, const int32_t* __restrict__ hist, int32_t* __restrict__ sorted_token,
                           int32_t* __restrict__ inv_pos, int32_t* __restrict__ group_sizes,
                           int32_t* __restrict__ group_offsets, const __nv_bfloat16* __restrict__ w,
                           float* __restrict__ sorted_w, int32_t* __restrict__ active) {
  extern __shared__ int sm[];
  constexpr int kWarps = kPermThreads / 32;
  int* base = sm;
  int* goff = sm + E;
  int* run = sm + 2 * E;
  int* wcnt = sm + 3 * E;
  __shared__ int carry_sh, active_sh;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int b = blockIdx.x, nblk = gridDim.x;

  // Expert totals, this block's base, and the expert offsets (block 0 also
  // lists the experts that kept rows, in order, when `active` is given).
  if (threadIdx.x == 0) carry_sh = active_sh = 0;
  __syncthreads();
  for (int e0 = 0; e0 < E; e0 += blockDim.x) {
    const int e = e0 + threadIdx.x;
    int kept = 0;
    if (e < E) {
      int pre = 0, tot = 0;
      for (int bb = 0; bb < nblk; ++bb) {
        const int h = hist[bb * E + e];
        pre += (bb < b) ? h : 0;
        tot += h;
      }
      base[e] = pre;
      run[e] = 0;
      kept = capacity >= 0 ? min(tot, capacity) : tot;
      for (int ww = 0; ww < kWarps; ++ww) wcnt[ww * E + e] = 0;
    }
    int total;
    const int off = block_exclusive_scan(kept, &total);
    const int carry = carry_sh;
    if (e < E) {
      goff[e] = carry + off;
      if (b == 0) {
        group_sizes[e] = kept;
        group_offsets[e] = carry + off;
      }
    }
    if (b == 0 && active != nullptr) {  // uniform over the block
      int n_active;
      const int pos = block_exclusive_scan((e < E && kept > 0) ? 1 : 0, &n_active);
      if (e < E && kept > 0) active[1 + active_sh + pos] = e;
      __syncthreads();
      if (threadIdx.x == 0) active_sh += n_active;
    }
    __syncthreads();
    if (threadIdx.x == 0) carry_sh = carry + total;
    __syncthreads();
  }
  if (b == 0 && threadIdx.x == 0) {
    group_offsets[E] = carry_sh;
    if (active != nullptr) active[0] = active_sh;
  }

  const int beg = b * chunk;
  const int end = min(m, beg + chunk);
  for (int r0 = beg; r0 < end; r0 += blockDim.x) {
    const int i = r0 + threadIdx.x;
    int e = (i < end) ? idx[i] : -1;
    if (e >= E || e < 0) e = -1;
    const float wv = (e >= 0 && sorted_w != nullptr) ? __bfloat162float(w[i]) : 0.f;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int lrank = __popc(peers & ((1u << lane) - 1u));
    const bool leader = lrank == 0;
    if (e >= 0 && leader) wcnt[warp * E + e] = __popc(peers);
    __syncthreads();
    if (e >= 0) {
      int slot = base[e] + run[e] + lrank;
      for (int ww = 0; ww < warp; ++ww) slot += wcnt[ww * E + e];
      if (capacity < 0 || slot < capacity) {
        const int p = goff[e] + slot;
        sorted_token[p] = i / k;
        inv_pos[i] = p;
        if (sorted_w != nullptr) sorted_w[p] = wv;
      } else {
        inv_pos[i] = -1;
      }
    } else if (i < end) {
      inv_pos[i] = -1;
    }
    __syncthreads();
    if (e >= 0 && leader) {
      wcnt[warp * E + e] = 0;
      atomicAdd(&run[e], __popc(peers));
    }
    __syncthreads();
  }
}

// Tile table: every group's rows cut into ceil(n / nt) runs of near-equal
// length (at most `nt` rows each).
__global__ void __launch_bounds__(kBlock, 1)
    build_tiles_kernel(const int32_t* __restrict__ group_offsets, int E, int nt,
                       TileEntry* __restrict__ tiles, int32_t* __restrict__ num_tiles) {
  __shared__ int carry_sh;
  if (threadIdx.x == 0) carry_sh = 0;
  __syncthreads();
  for (int e0 = 0; e0 < E; e0 += kBlock) {
    const int e = e0 + threadIdx.x;
    int n = 0, start = 0;
    if (e < E) {
      start = group_offsets[e];
      n = group_offsets[e + 1] - start;
    }
    const int cnt = (n + nt - 1) / nt;
    int tot;
    const int off = block_exclusive_scan(cnt, &tot) + carry_sh;
    // Balanced split: tile j covers rows [n*j/cnt, n*(j+1)/cnt), <= nt each.
    for (int j = 0; j < cnt; ++j) {
      const int lo = static_cast<int>(static_cast<int64_t>(n) * j / cnt);
      const int hi = static_cast<int>(static_cast<int64_t>(n) * (j + 1) / cnt);
      TileEntry te;
      te.group = e;
      te.row0 = start + lo;
      te.nrows = hi - lo;
      te.pad = 0;
      tiles[off + j] = te;
    }
    __syncthreads();
    if (threadIdx.x == 0) carry_sh += tot;
    __syncthreads();
  }
  if (threadIdx.x == 0) *num_tiles = carry_sh;
}

// ----------------------------------------------------------- gather ----
// xs[p] = x[sorted_token[p]] for p < min(*total_rows, max_rows) (all
// max_rows rows when total_rows is null); 16-byte vectors.
__global__ void gather_rows_kernel(const uint4* __restrict__ x, const int32_t* __restrict__ sorted_token,
                                   const int32_t* __restrict__ total_rows, int64_t max_rows,
                                   int vec_per_row, uint4* __restrict__ xs) {
  const int64_t tr = total_rows != nullptr ? *total_rows : max_rows;
  const int64_t rows = tr < max_rows ? tr : max_rows;
  const int64_t n = rows * vec_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / vec_per_row;
    const int c = static_cast<int>(i - r * vec_per_row);
    xs[i] = x[static_cast<int64_t>(sorted_token[r]) * vec_per_row + c];
  }
}

// ---------------------------------------------------------- combine ----
// Σ_j f32(w[t][j]) * f32(ys[inv_pos[t*k+j]][8c..8c+7]) in slot order j, as
// bf16 (out_f32 == 0) or fp32 (out_f32 == 1) into row t of out.
__global__ void combine_kernel(const uint4* __restrict__ ys, const int32_t* __restrict__ inv_pos,
                               const __nv_bfloat16* __restrict__ w, int64_t T, int k,
                               int vec_per_row, int out_f32, void* __restrict__ out) {
  const int64_t n = T * vec_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / vec_per_row;
    const int c = static_cast<int>(i - t * vec_per_row);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int p = inv_pos[t * k + j];
      if (p < 0) continue;
      const float wj = __bfloat162float(w[t * k + j]);
      const uint4 v = ys[static_cast<int64_t>(p) * vec_per_row + c];
      const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] = fmaf(wj, __uint_as_float(words[q] << 16), acc[2 * q]);
        acc[2 * q + 1] = fmaf(wj, __uint_as_float(words[q] & 0xFFFF0000u), acc[2 * q + 1]);
      }
    }
    if (out_f32) {
      float4* o = static_cast<float4*>(out) + 2 * i;
      o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
      continue;
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * q], acc[2 * q + 1]);
      ow[q] = *reinterpret_cast<const uint32_t*>(&b);
    }
    static_cast<uint4*>(out)[i] = o;
  }
}

// out[i] = bf16(acc[i]) for the fp32 accumulation of the fused combine.
__global__ void f32_to_bf16_kernel(const float4* __restrict__ acc, int64_t n4,
                                   uint2* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 v = acc[i];
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t*>(&a);
    o.y = *reinterpret_cast<const uint32_t*>(&b);
    out[i] = o;
  }
}

int grid_for(int64_t n, int threads, int cap) {
  int64_t g = (n + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return static_cast<int>(g);
}

}  // namespace

int launch_topk(const float* logits, int64_t T, int64_t E, int k, int32_t* idx, void* w,
                cudaStream_t stream, float* zero_rows, int64_t zero_cols) {
  KW8_REQUIRE(zero_rows == nullptr ||
                  (zero_cols % 4 == 0 && (reinterpret_cast<uintptr_t>(zero_rows) & 15) == 0),
              KW8_ERR_UNSUPPORTED, "rows to zero need 4-float alignment");
  KW8_REQUIRE(E >= 1 && E <= 32 * kMaxPerLane, KW8_ERR_UNSUPPORTED,
              "top-k supports 1..%d experts (got %lld)", 32 * kMaxPerLane, (long long)E);
  KW8_REQUIRE(k >= 1 && k <= 32 && k <= E, KW8_ERR_INVALID_ARG, "k=%d invalid for E=%lld", k,
              (long long)E);
  if (T <= 0) return KW8_OK;
  const int warps = 8;
  const int64_t blocks = (T + warps - 1) / warps;
  KW8_REQUIRE(blocks < (1ll << 31), KW8_ERR_UNSUPPORTED, "too many tokens");
  topk_softmax_kernel<<<static_cast<unsigned>(blocks), warps * 32, 0, stream>>>(
      logits, static_cast<int>(T), static_cast<int>(E), k, idx, static_cast<__nv_bfloat16*>(w),
      reinterpret_cast<float4*>(zero_rows), static_cast<int>(zero_cols / 4));
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_route_tail_small(const float* logits, int64_t T, int64_t E, int k, int64_t capacity,
                            int32_t* idx, void* w, int32_t* sorted_token, int32_t* inv_pos,
                            int32_t* group_sizes, int32_t* group_offsets, float* sorted_w,
                            int32_t* active, float* zero_rows, int64_t zero_cols,
                            cudaStream_t stream) {
  KW8_REQUIRE(route_tail_small_ok(T, E, k), KW8_ERR_UNSUPPORTED,
              "small routing tail: T*k <= %d and E <= %d (got T=%lld E=%lld k=%d)", kTailMaxRows,
              kTailThreads, (long long)T, (long long)E, k);
  KW8_REQUIRE(w && sorted_w && active, KW8_ERR_INVALID_ARG, "null routing output");
  KW8_REQUIRE(zero_rows == nullptr ||
                  (zero_cols % 4 == 0 && (reinterpret_cast<uintptr_t>(zero_rows) & 15) == 0),
              KW8_ERR_UNSUPPORTED, "rows to zero need 4-float alignment");
  const int cap = capacity < 0 ? -1 : static_cast<int>(std::min<int64_t>(capacity, 1ll << 30));
  route_tail_small_kernel<<<1, kTailThreads, 0, stream>>>(
      logits, static_cast<int>(T), static_cast<int>(E), k, cap, idx,
      static_cast<__nv_bfloat16*>(w), sorted_token, inv_pos, group_sizes, group_offsets, sorted_w,
      active, reinterpret_cast<float4*>(zero_rows), static_cast<int>(zero_cols / 4));
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_permute(const int32_t* idx, int64_t T, int k, int64_t E, int64_t capacity,
                   int32_t* sorted_token, int32_t* inv_pos, int32_t* group_sizes,
                   int32_t* group_offsets, cudaStream_t stream, const void* w,
                   float* sorted_w) {
  KW8_REQUIRE(E >= 1 && E <= 1024, KW8_ERR_UNSUPPORTED, "permute supports 1..1024 experts");
  KW8_REQUIRE(k >= 1 && T >= 0 && T * k < (1ll << 31), KW8_ERR_INVALID_ARG, "bad T/k");
  const int m = static_cast<int>(T * k);
  const int cap = capacity < 0 ? -1 : static_cast<int>(std::min<int64_t>(capacity, 1ll << 30));
  const size_t smem = static_cast<size_t>(33) * E * sizeof(int);
  static bool attr_set[64] = {false};
  int dev = 0;
  KW8_CUDA_TRY(cudaGetDevice(&dev));
  if (smem > 48 * 1024 && dev >= 0 && dev < 64 && !attr_set[dev]) {
    KW8_CUDA_TRY(cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(33 * 1024 * sizeof(int))));
    attr_set[dev] = true;
  }
  permute_kernel<<<1, kBlock, smem, stream>>>(idx, m, k, static_cast<int>(E), cap, sorted_token,
                                              inv_pos, group_sizes, group_offsets,
                                              static_cast<const __nv_bfloat16*>(w), sorted_w);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int64_t permute_hist_ints(int64_t E) { return static_cast<int64_t>(kPermMaxBlocks) * E; }

int launch_permute_multi(const int32_t* idx, int64_t T, int k, int64_t E, int64_t capacity,
                         int32_t* hist, int32_t* sorted_token, int32_t* inv_pos,
                         int32_t* group_sizes, int32_t* group_offsets, cudaStream_t stream,
                         const void* w, float* sorted_w, int32_t* active) {
  KW8_REQUIRE(E >= 1 && E <= 1024, KW8_ERR_UNSUPPORTED, "permute supports 1..1024 experts");
  KW8_REQUIRE(k >= 1 && T >= 0 && T * k < (1ll << 31), KW8_ERR_INVALID_ARG, "bad T/k");
  const int m = static_cast<int>(T * k);
  const int cap = capacity < 0 ? -1 : static_cast<int>(std::min<int64_t>(capacity, 1ll << 30));
  // Blocks of whole 256-entry rounds, at most kPermMaxBlocks of them.
  int nblk = std::max(1, std::min(kPermMaxBlocks, (m + kPermThreads - 1) / kPermThreads));
  int chunk = (m + nblk - 1) / nblk;
  chunk = (chunk + kPermThreads - 1) / kPermThreads * kPermThreads;
  if (chunk == 0) chunk = kPermThreads;
  nblk = std::max(1, (m + chunk - 1) / chunk);
  const size_t smem1 = static_cast<size_t>(E) * sizeof(int);
  const size_t smem2 = static_cast<size_t>(3 + kPermThreads / 32) * E * sizeof(int);
  static bool attr_set[64] = {false};
  int dev = 0;
  KW8_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    KW8_CUDA_TRY(cudaFuncSetAttribute(permute_scatter_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>((3 + kPermThreads / 32) * 1024 * sizeof(int))));
    attr_set[dev] = true;
  }
  permute_hist_kernel<<<nblk, kPermThreads, smem1, stream>>>(idx, m, static_cast<int>(E), chunk, hist);
  KW8_CHECK_LAUNCH();
  permute_scatter_kernel<<<nblk, kPermThreads, smem2, stream>>>(
      idx, m, k, static_cast<int>(E), cap, chunk, hist, sorted_token, inv_pos, group_sizes,
      group_offsets, static_cast<const __nv_bfloat16*>(w), sorted_w, active);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_build_tiles(const int32_t* group_offsets, int64_t E, int nt, TileEntry* tiles,
                       int32_t* num_tiles, cudaStream_t stream) {
  KW8_REQUIRE(E >= 1 && E <= (1 << 20) && nt >= 1, KW8_ERR_INVALID_ARG, "bad tile table args");
  build_tiles_kernel<<<1, kBlock, 0, stream>>>(group_offsets, static_cast<int>(E), nt, tiles,
                                               num_tiles);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_gather(const void* x, const int32_t* sorted_token, const int32_t* total_rows,
                  int64_t max_rows, int64_t D, void* xs, cudaStream_t stream) {
  KW8_REQUIRE(D % 8 == 0, KW8_ERR_UNSUPPORTED, "D must be a multiple of 8");
  if (max_rows <= 0) return KW8_OK;
  const int vec = static_cast<int>(D / 8);
  gather_rows_kernel<<<grid_for(max_rows * vec, 256, 148 * 16), 256, 0, stream>>>(
      static_cast<const uint4*>(x), sorted_token, total_rows, max_rows, vec,
      static_cast<uint4*>(xs));
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_combine(const void* ys, const int32_t* inv_pos, const void* w, int64_t T, int k,
                   int64_t D, void* out, cudaStream_t stream, bool out_f32) {
  KW8_REQUIRE(D % 8 == 0, KW8_ERR_UNSUPPORTED, "D must be a multiple of 8");
  if (T <= 0) return KW8_OK;
  const int vec = static_cast<int>(D / 8);
  combine_kernel<<<grid_for(T * vec, 256, 148 * 16), 256, 0, stream>>>(
      static_cast<const uint4*>(ys), inv_pos, static_cast<const __nv_bfloat16*>(w), T, k, vec,
      out_f32 ? 1 : 0, out);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_f32_to_bf16(const float* acc, int64_t n, void* out, cudaStream_t stream) {
  KW8_REQUIRE(n % 4 == 0, KW8_ERR_UNSUPPORTED, "element count must be a multiple of 4");
  if (n <= 0) return KW8_OK;
  f32_to_bf16_kernel<<<grid_for(n / 4, 256, 148 * 16), 256, 0, stream>>>(
      reinterpret_cast<const float4*>(acc), n / 4, static_cast<uint2*>(out));
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

}  // namespace kw8
