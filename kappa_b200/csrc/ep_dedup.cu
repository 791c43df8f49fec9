// Expert-parallel MoE step with each token sent once per owning rank.
//
// A token routed to several experts of one rank crosses NVLink once, not
// once per expert (with k = 8 of 128 experts on 2 ranks a token reaches
// both ranks but is routed 8 times).  Per call, on a source rank s:
//   * tok_slot[t][r] numbers the tokens that rank r needs (any kept routed
//     slot of t on an expert r owns), in token order; u[s][r] is their count;
//   * rows: token t goes to rank r's row buffer at uoff(r, s) + slot, with
//     uoff(r, s) = sum_{s' < s} u[s'][r] (source-major);
//   * pair records: routed pair p of expert e (kept, sorted order) goes to
//     e's owner r at the pair's place in r's expert-major layout
//     (recv_pos, as in ep.cu): {its token's row index on r, its weight}.
// On an owner rank r: the pairs' rows are gathered locally into expert
// order, the expert FFN runs on them and its down projection adds w * y
// into one fp32 partial row per received token (the fused combine, rows
// indexed by the records); each partial goes back to its source as bf16
// (ret[r][slot] on the source), and the source sums its partials over the
// ranks in rank order.  The partials travel as fp32 (the sum is rounded
// once, as on one GPU), as fp16 with a per-row power-of-two scale (half the
// traffic, relative error per partial up to 2^-11) or as bf16 (half the
// traffic, up to 2^-9).
#include "ep.cuh"

namespace kw8 {

namespace {

constexpr int kDdThreads = 256;
constexpr int kCopyBatch = 8;  // 16-byte chunks a lane loads before storing them to a peer

// tok_slot[t][r] and u_cnt[r] (see above).  One CTA of 1024 threads.
__global__ void __launch_bounds__(1024)
    ep_slots_kernel(const int32_t* __restrict__ idx, const int32_t* __restrict__ inv_pos, int T, int k, int El,
                    int world, int32_t* __restrict__ tok_slot, int32_t* __restrict__ u_cnt) {
  __shared__ int carry[kEpMaxRanks];
  if (threadIdx.x < kEpMaxRanks) carry[threadIdx.x] = 0;
  __syncthreads();
  for (int t0 = 0; t0 < T; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    unsigned mask = 0;
    if (t < T)
      for (int j = 0; j < k; ++j)
        if (inv_pos[static_cast<int64_t>(t) * k + j] >= 0) mask |= 1u << (idx[static_cast<int64_t>(t) * k + j] / El);
    for (int r = 0; r < world; ++r) {
      const int flag = static_cast<int>((mask >> r) & 1u);
      int total;
      const int pos = block_exclusive_scan(flag, &total);
      if (t < T) tok_slot[static_cast<int64_t>(t) * world + r] = flag ? carry[r] + pos : -1;
      __syncthreads();
      if (threadIdx.x == 0) carry[r] += total;
      __syncthreads();
    }
  }
  if (threadIdx.x < world) u_cnt[threadIdx.x] = carry[threadIdx.x];
}

// Counts row of this rank (E expert counts, then world unique-token counts)
// into every rank's counts[epoch & 1], then phase 0 of the group flags.
__global__ void ep_counts2_kernel(const int32_t* __restrict__ sizes, const int32_t* __restrict__ u_cnt, int E,
                                  const uint64_t* __restrict__ counts, const uint64_t* __restrict__ flags,
                                  uint32_t* own_flags, int world, int rank, uint32_t epoch) {
  const int parity = static_cast<int>(epoch & 1u);
  const int row = E + world;
  for (int p = 0; p < world; ++p) {
    int32_t* dst = reinterpret_cast<int32_t*>(counts[p]) + (static_cast<int64_t>(parity) * world + rank) * row;
    for (int i = threadIdx.x; i < row; i += blockDim.x) dst[i] = i < E ? sizes[i] : u_cnt[i - E];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world) flag_release(reinterpret_cast<uint32_t*>(flags[threadIdx.x]) + rank, epoch);
  if (threadIdx.x < world) flag_wait(own_flags + threadIdx.x, epoch);
  __syncthreads();
}

// Token rows (a warp per token) and pair records (a thread per pair) to
// their owners.  counts: this call's rows (stride E + world).
__global__ void __launch_bounds__(kDdThreads)
    ep_dispatch2_kernel(const uint4* __restrict__ x, int vec, int T, const int32_t* __restrict__ sorted_token,
                        const int32_t* __restrict__ offsets, const float* __restrict__ sorted_w,
                        const int32_t* __restrict__ tok_slot, const int32_t* __restrict__ counts, int world,
                        int rank, int E, int El, int64_t pair_cap, const uint64_t* __restrict__ peer_rows,
                        const uint64_t* __restrict__ peer_meta) {
  extern __shared__ int sh[];
  int* off = sh;               // [E+1] this rank's expert offsets
  int* dest = sh + E + 1;      // [E]   recv_pos(rank, e, 0) on e's owner
  int* uoff = sh + 2 * E + 1;  // [world] this rank's first row on rank r
  const int cs = E + world;
  for (int e = threadIdx.x; e <= E; e += blockDim.x) off[e] = offsets[e];
  recv_bases(counts, cs, world, E, El, rank, dest);
  for (int r = threadIdx.x; r < world; r += blockDim.x) {
    int acc = 0;
    for (int s = 0; s < rank; ++s) acc += counts[s * cs + E + r];
    uoff[r] = acc;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int t = blockIdx.x * wpb + (threadIdx.x >> 5); t < T; t += gridDim.x * wpb) {
    const uint4* src = x + static_cast<int64_t>(t) * vec;
    for (int c0 = 0; c0 < vec; c0 += 32 * kCopyBatch) {
      // This lane's chunks of the row in registers first, so the loads are
      // in flight together (the peer stores may alias them for the compiler).
      uint4 v[kCopyBatch];
#pragma unroll
      for (int j = 0; j < kCopyBatch; ++j) {
        const int c = c0 + j * 32 + lane;
        if (c < vec) v[j] = __ldg(src + c);
      }
      for (int r = 0; r < world; ++r) {
        const int slot = tok_slot[static_cast<int64_t>(t) * world + r];
        if (slot < 0) continue;  // uniform over the warp
        uint4* dst = reinterpret_cast<uint4*>(peer_rows[r]) + static_cast<int64_t>(uoff[r] + slot) * vec;
#pragma unroll
        for (int j = 0; j < kCopyBatch; ++j) {
          const int c = c0 + j * 32 + lane;
          if (c < vec) dst[c] = v[j];
        }
      }
    }
  }
  const int pairs = off[E];
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < pairs; p += gridDim.x * blockDim.x) {
    const int e = upper_index(off, E + 1, p);
    const int r = e / El;
    const int pos = dest[e] + (p - off[e]);
    const int t = sorted_token[p];
    int32_t* meta = reinterpret_cast<int32_t*>(peer_meta[r]);
    meta[pos] = uoff[r] + tok_slot[static_cast<int64_t>(t) * world + r];
    reinterpret_cast<float*>(meta + pair_cap)[pos] = sorted_w[p];
  }
  __threadfence_system();
}

// Owner side: xs[pos] = rows[meta[pos]] for every received pair (a warp
// per pair), and the fp32 partial rows P[0 .. received tokens) zeroed.
__global__ void __launch_bounds__(kDdThreads)
    ep_gather2_kernel(const uint4* __restrict__ rows, const int32_t* __restrict__ meta,
                      const int32_t* __restrict__ loc_off, int El, const int32_t* __restrict__ counts, int world,
                      int rank, int E, int vec, uint4* __restrict__ xs, float4* __restrict__ part, int D) {
  const int pairs = loc_off[El];
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int q = blockIdx.x * wpb + (threadIdx.x >> 5); q < pairs; q += gridDim.x * wpb) {
    const uint4* src = rows + static_cast<int64_t>(meta[q]) * vec;
    uint4* dst = xs + static_cast<int64_t>(q) * vec;
    for (int c = lane; c < vec; c += 32) dst[c] = src[c];
  }
  int utot = 0;
  for (int s = 0; s < world; ++s) utot += counts[s * (E + world) + E + rank];
  const int64_t n4 = static_cast<int64_t>(utot) * (D / 4);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    part[i] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// Owner side: partial row u (source s, slot u - uoff(rank, s)) into source
// s's return buffer at [rank][slot], in the group's return format:
//   KW8_RET_F32        fp32 as computed;
//   KW8_RET_BF16       bf16 (one rounding, relative error up to 2^-9);
//   KW8_RET_F16_SCALED fp16 of the row divided by a power of two 2^(e-14),
//                      e = floor(log2 max|row|), so every value is a normal
//                      fp16 (relative error up to 2^-11) at bf16's size; the
//                      scale goes to the return buffer's scale array.
// A warp per row.
__global__ void __launch_bounds__(kDdThreads)
    ep_return2_kernel(const float4* __restrict__ part, int D, const int32_t* __restrict__ counts, int world,
                      int rank, int E, int64_t max_tokens, const uint64_t* __restrict__ peer_ret, int fmt) {
  __shared__ int start[kEpMaxRanks + 1];  // first row of each source
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int s = 0; s < world; ++s) {
      start[s] = acc;
      acc += counts[s * (E + world) + E + rank];
    }
    start[world] = acc;
  }
  __syncthreads();
  const int rows = start[world];
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int v8 = D / 8;  // 8 values per lane step
  for (int u = blockIdx.x * wpb + (threadIdx.x >> 5); u < rows; u += gridDim.x * wpb) {
    int s = 0;
    while (s + 1 < world && start[s + 1] <= u) ++s;
    const float4* src = part + static_cast<int64_t>(u) * (D / 4);
    const int64_t drow = static_cast<int64_t>(rank) * max_tokens + (u - start[s]);
    if (fmt == KW8_RET_F32) {
      // Loads of a batch in registers first, then the peer stores (they
      // may alias for the compiler, which would otherwise serialise them).
      float4* dst = reinterpret_cast<float4*>(peer_ret[s]) + drow * (D / 4);
      for (int c0 = 0; c0 < D / 4; c0 += 32 * kCopyBatch) {
        float4 v[kCopyBatch];
#pragma unroll
        for (int j = 0; j < kCopyBatch; ++j) {
          const int c = c0 + j * 32 + lane;
          if (c < D / 4) v[j] = src[c];
        }
#pragma unroll
        for (int j = 0; j < kCopyBatch; ++j) {
          const int c = c0 + j * 32 + lane;
          if (c < D / 4) dst[c] = v[j];
        }
      }
      continue;
    }
    float inv = 1.0f;  // 1 / scale (KW8_RET_F16_SCALED)
    if (fmt == KW8_RET_F16_SCALED) {
      float m = 0.f;
      for (int c = lane; c < D / 4; c += 32) {
        const float4 a = src[c];
        m = fmaxf(m, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      int e = 0;
      if (m > 0.f && m <= 3.0e38f) e = max(ilogbf(m), -100);  // NaN / inf rows keep scale 1
      inv = ldexpf(1.0f, 14 - e);
      if (lane == 0) {
        float* scales = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(peer_ret[s]) +
                                                 static_cast<int64_t>(world) * max_tokens * D * 2);
        scales[drow] = ldexpf(1.0f, e - 14);
      }
    }
    uint4* dst = reinterpret_cast<uint4*>(peer_ret[s]) + drow * v8;
    for (int c0 = 0; c0 < v8; c0 += 32 * kCopyBatch) {
      uint4 o[kCopyBatch];
#pragma unroll
      for (int j = 0; j < kCopyBatch; ++j) {
        const int c = c0 + j * 32 + lane;
        if (c >= v8) continue;
        const float4 a = src[2 * c], b = src[2 * c + 1];
        uint32_t w[4];
        if (fmt == KW8_RET_F16_SCALED) {
          const __half2 h0 = __floats2half2_rn(a.x * inv, a.y * inv), h1 = __floats2half2_rn(a.z * inv, a.w * inv);
          const __half2 h2 = __floats2half2_rn(b.x * inv, b.y * inv), h3 = __floats2half2_rn(b.z * inv, b.w * inv);
          w[0] = *reinterpret_cast<const uint32_t*>(&h0);
          w[1] = *reinterpret_cast<const uint32_t*>(&h1);
          w[2] = *reinterpret_cast<const uint32_t*>(&h2);
          w[3] = *reinterpret_cast<const uint32_t*>(&h3);
        } else {
          const __nv_bfloat162 p0 = __floats2bfloat162_rn(a.x, a.y), p1 = __floats2bfloat162_rn(a.z, a.w);
          const __nv_bfloat162 p2 = __floats2bfloat162_rn(b.x, b.y), p3 = __floats2bfloat162_rn(b.z, b.w);
          w[0] = *reinterpret_cast<const uint32_t*>(&p0);
          w[1] = *reinterpret_cast<const uint32_t*>(&p1);
          w[2] = *reinterpret_cast<const uint32_t*>(&p2);
          w[3] = *reinterpret_cast<const uint32_t*>(&p3);
        }
        o[j] = make_uint4(w[0], w[1], w[2], w[3]);
      }
#pragma unroll
      for (int j = 0; j < kCopyBatch; ++j) {
        const int c = c0 + j * 32 + lane;
        if (c < v8) dst[c] = o[j];
      }
    }
  }
  __threadfence_system();
}

// Source side: out[t] = sum over ranks r (in order) of ret[r][tok_slot[t][r]]
// (partials in the group's return format) in fp32, then bf16 (zero for a
// token with no kept slot).  A warp per token.
__global__ void __launch_bounds__(kDdThreads)
    ep_final2_kernel(const void* __restrict__ ret, const int32_t* __restrict__ tok_slot, int T, int world,
                     int64_t max_tokens, int D, int fmt, uint4* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int v8 = D / 8;
  const float* scales =
      reinterpret_cast<const float*>(static_cast<const uint8_t*>(ret) + static_cast<int64_t>(world) * max_tokens * D * 2);
  for (int t = blockIdx.x * wpb + (threadIdx.x >> 5); t < T; t += gridDim.x * wpb) {
    for (int c = lane; c < v8; c += 32) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int r = 0; r < world; ++r) {
        const int slot = tok_slot[static_cast<int64_t>(t) * world + r];
        if (slot < 0) continue;
        const int64_t row = static_cast<int64_t>(r) * max_tokens + slot;
        if (fmt == KW8_RET_F32) {
          const float4* p = static_cast<const float4*>(ret) + row * (D / 4) + 2 * c;
          const float4 a = p[0], b = p[1];
          acc[0] += a.x; acc[1] += a.y; acc[2] += a.z; acc[3] += a.w;
          acc[4] += b.x; acc[5] += b.y; acc[6] += b.z; acc[7] += b.w;
          continue;
        }
        const uint4 v = static_cast<const uint4*>(ret)[row * v8 + c];
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
        if (fmt == KW8_RET_F16_SCALED) {
          const float sc = scales[row];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
            acc[2 * i] += f.x * sc;
            acc[2 * i + 1] += f.y * sc;
          }
          continue;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[2 * i] += __uint_as_float(w4[i] << 16);
          acc[2 * i + 1] += __uint_as_float(w4[i] & 0xFFFF0000u);
        }
      }
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
        o[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
      out[static_cast<int64_t>(t) * v8 + c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

int ep_grid(int64_t work, int per_block) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + per_block - 1) / per_block, 148 * 8)));
}

}  // namespace

int launch_ep_slots(const int32_t* idx, const int32_t* inv_pos, int64_t T, int k, int64_t E, int world,
                    int32_t* tok_slot, int32_t* u_cnt, cudaStream_t stream) {
  KW8_REQUIRE(world >= 1 && world <= kEpMaxRanks && E % world == 0, KW8_ERR_INVALID_ARG, "bad group");
  ep_slots_kernel<<<1, 1024, 0, stream>>>(idx, inv_pos, static_cast<int>(T), k, static_cast<int>(E / world),
                                           world, tok_slot, u_cnt);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_ep_counts2(const int32_t* sizes, const int32_t* u_cnt, int64_t E, const uint64_t* counts,
                      const uint64_t* flags, uint32_t* own_flags, int world, int rank, uint32_t epoch,
                      cudaStream_t stream) {
  ep_counts2_kernel<<<1, 256, 0, stream>>>(sizes, u_cnt, static_cast<int>(E), counts, flags, own_flags, world,
                                          rank, epoch);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_ep_dispatch2(const void* x, int64_t T, int k, int64_t D, const int32_t* sorted_token,
                        const int32_t* offsets, const float* sorted_w, const int32_t* tok_slot,
                        const int32_t* counts, int world, int rank, int64_t E, int64_t pair_cap,
                        const uint64_t* peer_rows, const uint64_t* peer_meta, cudaStream_t stream) {
  KW8_REQUIRE(D % 8 == 0, KW8_ERR_UNSUPPORTED, "D must be a multiple of 8");
  if (T <= 0) return KW8_OK;
  const size_t smem = (2 * static_cast<size_t>(E) + 1 + world) * sizeof(int);
  const int grid = std::max(ep_grid(T, kDdThreads / 32), ep_grid(T * k, kDdThreads));
  ep_dispatch2_kernel<<<grid, kDdThreads, smem, stream>>>(
      static_cast<const uint4*>(x), static_cast<int>(D / 8), static_cast<int>(T), sorted_token, offsets,
      sorted_w, tok_slot, counts, world, rank, static_cast<int>(E), static_cast<int>(E / world), pair_cap,
      peer_rows, peer_meta);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_ep_gather2(const void* rows, const int32_t* meta, const int32_t* loc_off, int64_t El,
                      const int32_t* counts, int world, int rank, int64_t E, int64_t D, int64_t max_pairs,
                      void* xs, float* part, cudaStream_t stream) {
  KW8_REQUIRE(D % 8 == 0, KW8_ERR_UNSUPPORTED, "D must be a multiple of 8");
  ep_gather2_kernel<<<ep_grid(max_pairs, kDdThreads / 32), kDdThreads, 0, stream>>>(
      static_cast<const uint4*>(rows), meta, loc_off, static_cast<int>(El), counts, world, rank,
      static_cast<int>(E), static_cast<int>(D / 8), static_cast<uint4*>(xs), reinterpret_cast<float4*>(part),
      static_cast<int>(D));
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_ep_return2(const float* part, int64_t D, const int32_t* counts, int world, int rank, int64_t E,
                      int64_t max_tokens, const uint64_t* peer_ret, int ret_format, cudaStream_t stream) {
  ep_return2_kernel<<<ep_grid(static_cast<int64_t>(world) * max_tokens, kDdThreads / 32), kDdThreads, 0,
                      stream>>>(reinterpret_cast<const float4*>(part), static_cast<int>(D), counts, world, rank,
                                static_cast<int>(E), max_tokens, peer_ret, ret_format);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_ep_final2(const void* ret, const int32_t* tok_slot, int64_t T, int world, int64_t max_tokens,
                     int64_t D, int ret_format, void* out, cudaStream_t stream) {
  if (T <= 0) return KW8_OK;
  ep_final2_kernel<<<ep_grid(T, kDdThreads / 32), kDdThreads, 0, stream>>>(
      ret, tok_slot, static_cast<int>(T), world, max_tokens, static_cast<int>(D), ret_format,
      static_cast<uint4*>(out));
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

}  // namespace kw8
