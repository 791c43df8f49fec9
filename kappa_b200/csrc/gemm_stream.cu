// Weight-streaming grouped W8A16 GEMM: kernel and launcher.  Design notes
// are in gemm_stream.cuh.
#include "gemm_stream.cuh"

namespace kw8 {

namespace {

constexpr int kStThreads = 256;  // 8 warps
constexpr int kStWarps = kStThreads / 32;
constexpr int kStStepK = 64;     // k per warp step: 4 lanes x 16 bytes
constexpr double kStCtaSteps = 3.0;  // fixed cost of a CTA, in warp steps (stream_plan)

// Per-warp copy ring: a stage holds one step's 16-byte chunks of every lane
// (kMats x 2 weight rows, 2 per 8-token tile).  Depth from the chunk count,
// so that two CTAs fit an SM where possible.
__host__ __device__ constexpr int stream_slots(bool pair, int nt) { return 2 * (pair ? 2 : 1) + 2 * (nt / 8); }
__host__ __device__ constexpr int stream_stages(int slots) { return slots <= 4 ? 6 : (slots <= 6 ? 4 : 3); }
__host__ __device__ constexpr int stream_smem_bytes(bool pair, int nt) {
  return kStWarps * stream_stages(stream_slots(pair, nt)) * stream_slots(pair, nt) * 32 * 16;
}

// 16-byte asynchronous copies global -> shared (this thread's own chunk);
// with src_bytes = 0 nothing is read and the destination is zero-filled.
// Weights bypass L1 (.cg: read once); token rows, which every warp of the
// CTA reads, are cached in L1 (.ca).
__device__ __forceinline__ void cp_async_cg16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_ca16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int kPending>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

__device__ __forceinline__ void mma_16816_bf16(float (&d)[4], uint32_t a0, uint32_t a1,
                                               uint32_t a2, uint32_t a3, uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 16 int8 (k0..k0+15) -> 8 bf16x2 words; word i holds k0 + 2i, k0 + 2i + 1.
__device__ __forceinline__ void widen16(const uint4& v, uint32_t (&a)[8]) {
  i8x4_to_bf16x4(v.x, a[0], a[1]);
  i8x4_to_bf16x4(v.y, a[2], a[3]);
  i8x4_to_bf16x4(v.z, a[4], a[5]);
  i8x4_to_bf16x4(v.w, a[6], a[7]);
}

template <int kMode, int kNT, bool kTiled>
__global__ void __launch_bounds__(kStThreads,
                                  stream_smem_bytes(epi_is_pair(kMode), kNT) <= 113 * 1024 ? 2 : 1)
    w8_stream_kernel(const int8_t* __restrict__ wa, const int8_t* __restrict__ wb,
                     const __nv_bfloat16* __restrict__ x, int64_t ldx, const StreamArgs p) {
  constexpr bool kPair = epi_is_pair(kMode);
  constexpr int kMats = kPair ? 2 : 1;
  constexpr int kNTiles = kNT / 8;
  constexpr int kAcc = kMats * kNTiles * 4;
  constexpr int kSlots = stream_slots(kPair, kNT);
  constexpr int kStages = stream_stages(kSlots);
  constexpr int kRingChunks = kStages * kSlots * 32;  // 16-byte chunks per warp
  static_assert(kAcc * 32 * 4 <= kRingChunks * 16, "partial sums reuse the ring");
  extern __shared__ uint4 stream_smem[];
  uint4* ring = stream_smem + (threadIdx.x >> 5) * kRingChunks;  // this warp's ring

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  int group = blockIdx.y;
  if (p.active_groups != nullptr) {
    if (group >= p.active_groups[0]) return;  // uniform over the CTA
    group = p.active_groups[1 + group];
  }
  int r_begin = 0, r_end = p.dense_rows;
  if (p.group_offsets != nullptr) {
    r_begin = p.group_offsets[group];
    r_end = p.group_offsets[group + 1];
  }
  // grid z = (K range kzi) x (row pass zi).
  const int kz = p.kz > 1 ? p.kz : 1;
  const int zc = static_cast<int>(gridDim.z) / kz;
  const int zi = static_cast<int>(blockIdx.z) % zc, kzi = static_cast<int>(blockIdx.z) / zc;
  // Same outcome for every thread of the CTA (no barrier has been passed).
  if (r_begin + zi * kNT >= r_end) return;

  const int ks = p.ks;
  const int ftile = blockIdx.x * (kStWarps / ks) + warp / ks;
  const int kslice = warp % ks;
  const int f0 = ftile * 16;
  const bool tile_ok = f0 < p.N_out;
  const int nsteps = (p.K + kStStepK - 1) / kStStepK;
  const int c_lo = nsteps * kzi / kz, c_hi = nsteps * (kzi + 1) / kz;  // this CTA's steps
  const int s_lo = c_lo + (c_hi - c_lo) * kslice / ks;
  const int s_hi = c_lo + (c_hi - c_lo) * (kslice + 1) / ks;

  // Feature rows g and g + 8 of the tile; rows past N_out read the last
  // row (a valid address) and are zeroed.
  const bool ok0 = f0 + g < p.N_out, ok1 = f0 + g + 8 < p.N_out;
  const int64_t wbase = static_cast<int64_t>(group) * p.N_out;
  const int64_t fr0 = wbase + min(f0 + g, p.N_out - 1);
  const int64_t fr1 = wbase + min(f0 + g + 8, p.N_out - 1);
  const int8_t* w_rows[kMats][2];
  if constexpr (kTiled) {
    // Block (group, ftile, step 0) of the tiled layout; lane (g, c) copies
    // its 16 bytes of row g at 16 (8 c + g) and of row g + 8 at 512 + that
    // (zeros past N and K are stored, so no fill is needed).  A step is
    // 1 KB further on: "k" below counts bytes of blocks, 64 per 1 KB.
    const int64_t blk_off =
        tile_ok ? (static_cast<int64_t>(group) * p.tile_ftiles + ftile) * p.tile_steps * kTiledBlock : 0;
    const int8_t* blk0 = wa + blk_off;
    w_rows[0][0] = blk0 + 16 * (8 * c + g);
    w_rows[0][1] = blk0 + 512 + 16 * (8 * c + g);
    if constexpr (kPair) {
      const int8_t* blk1 = wb + (blk0 - wa);
      w_rows[1][0] = blk1 + 16 * (8 * c + g);
      w_rows[1][1] = blk1 + 512 + 16 * (8 * c + g);
    }
  } else {
    w_rows[0][0] = wa + fr0 * p.K;
    w_rows[0][1] = wa + fr1 * p.K;
    if constexpr (kPair) {
      w_rows[1][0] = wb + fr0 * p.K;
      w_rows[1][1] = wb + fr1 * p.K;
    }
  }

  float s_a[2], s_b[2] = {0.f, 0.f};
  s_a[0] = load_scale(p.scale_a, p.scale_a_dtype, p.scale_a_pc ? fr0 : 0);
  s_a[1] = load_scale(p.scale_a, p.scale_a_dtype, p.scale_a_pc ? fr1 : 0);
  if constexpr (kPair) {
    s_b[0] = load_scale(p.scale_b, p.scale_b_dtype, p.scale_b_pc ? fr0 : 0);
    s_b[1] = load_scale(p.scale_b, p.scale_b_dtype, p.scale_b_pc ? fr1 : 0);
  }

  for (int row0 = r_begin + zi * kNT; row0 < r_end; row0 += zc * kNT) {
    const int nrows = min(kNT, r_end - row0);
    // Token row g of each 8-row tile; rows past nrows read row0 and are zeroed.
    const __nv_bfloat16* x_rows[kNTiles];
    bool x_ok[kNTiles];
#pragma unroll
    for (int t = 0; t < kNTiles; ++t) {
      x_ok[t] = t * 8 + g < nrows;
      const int r = row0 + (x_ok[t] ? t * 8 + g : 0);
      const int64_t xr = p.row_index != nullptr ? p.row_index[r] : r;
      x_rows[t] = x + xr * ldx;
    }
    float acc[kMats][kNTiles][4];
#pragma unroll
    for (int m = 0; m < kMats; ++m)
#pragma unroll
      for (int t = 0; t < kNTiles; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[m][t][e] = 0.f;

    if (tile_ok) {
      const int n = s_hi - s_lo;  // steps of this slice
      // The last step of K is partial when K % 64 != 0: its lanes past K
      // zero-fill from a clamped (valid) address.
      const int tail_j = (p.K % kStStepK != 0 && s_hi == nsteps) ? n - 1 : -1;
      // Tiled weights store zeros past N: every row copies.
      const uint32_t wn0 = (kTiled || ok0) ? 16u : 0u, wn1 = (kTiled || ok1) ? 16u : 0u;
      // Bytes between consecutive steps of a weight row, and the first.
      constexpr int kWStep = kTiled ? kTiledBlock : kStStepK;
      uint32_t xn[kNTiles];
#pragma unroll
      for (int t = 0; t < kNTiles; ++t) xn[t] = x_ok[t] ? 16u : 0u;
      // Running pointers at step j0 of the slice (this lane's 16 k included);
      // within an unrolled round every copy is at an immediate offset.
      const int k_first = s_lo * kStStepK + c * 16;
      const int8_t* wp[kMats][2];
      const __nv_bfloat16* xp[kNTiles];
      const int64_t w_first = kTiled ? static_cast<int64_t>(s_lo) * kTiledBlock : k_first;
#pragma unroll
      for (int m = 0; m < kMats; ++m) {
        wp[m][0] = w_rows[m][0] + w_first;
        wp[m][1] = w_rows[m][1] + w_first;
      }
#pragma unroll
      for (int t = 0; t < kNTiles; ++t) xp[t] = x_rows[t] + k_first;
      uint4* const rl = ring + lane;
      // Step j (= j0 + off) into ring stage st.
      auto issue = [&](int j, int off, int st) {
        uint4* dst = rl + st * kSlots * 32;
        if (j != tail_j) {
#pragma unroll
          for (int m = 0; m < kMats; ++m) {
            cp_async_cg16(dst + (2 * m) * 32, wp[m][0] + off * kWStep, wn0);
            cp_async_cg16(dst + (2 * m + 1) * 32, wp[m][1] + off * kWStep, wn1);
          }
#pragma unroll
          for (int t = 0; t < kNTiles; ++t) {
            cp_async_ca16(dst + (2 * kMats + 2 * t) * 32, xp[t] + off * kStStepK, xn[t]);
            cp_async_ca16(dst + (2 * kMats + 2 * t + 1) * 32, xp[t] + off * kStStepK + 8, xn[t]);
          }
        } else {
          // Lanes past K read the row's last 16 k instead (shifted back by
          // `back`) and zero-fill.
          const int kc = k_first + j * kStStepK;
          const bool kok = kc < p.K;
          const int back = kok ? 0 : kc - (p.K - 16);
          const int o = off * kStStepK - back;
#pragma unroll
          for (int m = 0; m < kMats; ++m) {
            if constexpr (kTiled) {  // the block holds zeros past K
              cp_async_cg16(dst + (2 * m) * 32, wp[m][0] + off * kWStep, wn0);
              cp_async_cg16(dst + (2 * m + 1) * 32, wp[m][1] + off * kWStep, wn1);
            } else {
              cp_async_cg16(dst + (2 * m) * 32, wp[m][0] + o, kok ? wn0 : 0u);
              cp_async_cg16(dst + (2 * m + 1) * 32, wp[m][1] + o, kok ? wn1 : 0u);
            }
          }
#pragma unroll
          for (int t = 0; t < kNTiles; ++t) {
            cp_async_ca16(dst + (2 * kMats + 2 * t) * 32, xp[t] + o, kok ? xn[t] : 0u);
            cp_async_ca16(dst + (2 * kMats + 2 * t + 1) * 32, xp[t] + o + 8, kok ? xn[t] : 0u);
          }
        }
      };
      // Ring of kStages steps: kStages - 1 copy groups in flight ahead of
      // the step being multiplied; step j lives in stage j % kStages.  Each
      // lane reads back only the chunks it copied, so its own wait_group is
      // the only synchronisation.
#pragma unroll
      for (int d = 0; d < kStages - 1; ++d) {
        if (d < n) issue(d, d, d);
        cp_async_commit();
      }
      for (int j0 = 0; j0 < n; j0 += kStages) {
#pragma unroll
        for (int d = 0; d < kStages; ++d) {
          if (j0 + d < n) {
            // The step kStages - 1 ahead goes into the stage step j0 + d - 1 freed.
            if (j0 + d + kStages - 1 < n) issue(j0 + d + kStages - 1, d + kStages - 1, (d + kStages - 1) % kStages);
            cp_async_commit();
            cp_async_wait<kStages - 1>();
            const uint4* src = rl + d * kSlots * 32;
            uint32_t a[kMats][2][8];
#pragma unroll
            for (int m = 0; m < kMats; ++m) {
              widen16(src[(2 * m) * 32], a[m][0]);
              widen16(src[(2 * m + 1) * 32], a[m][1]);
            }
#pragma unroll
            for (int t = 0; t < kNTiles; ++t) {
              const uint4 x0 = src[(2 * kMats + 2 * t) * 32];
              const uint4 x1 = src[(2 * kMats + 2 * t + 1) * 32];
              const uint32_t xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
              for (int q = 0; q < 4; ++q)
#pragma unroll
                for (int m = 0; m < kMats; ++m)
                  mma_16816_bf16(acc[m][t], a[m][0][2 * q], a[m][1][2 * q], a[m][0][2 * q + 1],
                                 a[m][1][2 * q + 1], xw[2 * q], xw[2 * q + 1]);
            }
          }
        }
#pragma unroll
        for (int m = 0; m < kMats; ++m) {
          wp[m][0] += kStages * kWStep;
          wp[m][1] += kStages * kWStep;
        }
#pragma unroll
        for (int t = 0; t < kNTiles; ++t) xp[t] += kStages * kStStepK;
      }
    }

    // K slices meet in shared memory (each warp's own ring, idle now: its
    // last real copy group has been waited for); slice 0 adds the others in
    // order.
    if (ks > 1) {
      float* red = reinterpret_cast<float*>(ring);  // [kAcc][32] of this warp
      if (kslice != 0) {
#pragma unroll
        for (int m = 0; m < kMats; ++m)
#pragma unroll
          for (int t = 0; t < kNTiles; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) red[((m * kNTiles + t) * 4 + e) * 32 + lane] = acc[m][t][e];
      }
      __syncthreads();
      if (kslice == 0) {
        for (int j = 1; j < ks; ++j) {
          const float* other = reinterpret_cast<const float*>(ring + j * kRingChunks);
#pragma unroll
          for (int m = 0; m < kMats; ++m)
#pragma unroll
            for (int t = 0; t < kNTiles; ++t)
#pragma unroll
              for (int e = 0; e < 4; ++e) acc[m][t][e] += other[((m * kNTiles + t) * 4 + e) * 32 + lane];
        }
      }
      __syncthreads();
    }
    if (kslice != 0 || !tile_ok) continue;

    // acc[m][t][e]: feature f0 + g + 8 (e / 2), token t * 8 + 2c + (e % 2).
#pragma unroll
    for (int t = 0; t < kNTiles; ++t) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hi = e >> 1;
        const int f = f0 + g + 8 * hi;
        const int tt = t * 8 + 2 * c + (e & 1);
        if (f >= p.N_out || tt >= nrows) continue;
        const int row = row0 + tt;
        const float y = acc[0][t][e] * s_a[hi];
        if constexpr (kPair) {
          const float u = acc[kMats - 1][t][e] * s_b[hi];
          const float h = (kMode == EPI_PAIR_GELU) ? gelu_tanh_f(y) * u : silu_f(y) * u;
          static_cast<__nv_bfloat16*>(p.out)[static_cast<int64_t>(row) * p.ld_out + f] =
              __float2bfloat16_rn(h);
        } else if constexpr (kMode == EPI_COMBINE_F32) {
          atomicAdd(static_cast<float*>(p.out) + static_cast<int64_t>(p.row_token[row]) * p.ld_out + f,
                    y * p.row_weight[row]);
        } else if constexpr (kMode == EPI_PLAIN_F32) {
          static_cast<float*>(p.out)[kzi * p.split_stride + static_cast<int64_t>(row) * p.ld_out + f] = y;
        } else {
          static_cast<__nv_bfloat16*>(p.out)[static_cast<int64_t>(row) * p.ld_out + f] =
              __float2bfloat16_rn(y);
        }
      }
    }
  }
}

template <int kMode, int kNT, bool kTiled>
int launch_stream_nt(dim3 grid, const int8_t* wa, const int8_t* wb, const void* x, int64_t ldx,
                     const StreamArgs& a, cudaStream_t stream) {
  constexpr int smem = stream_smem_bytes(epi_is_pair(kMode), kNT);
  static_assert(smem <= kTcDynSmemMax, "copy ring exceeds shared memory");
  static bool attr_set[64] = {false};
  int dev = 0;
  KW8_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    KW8_CUDA_TRY(cudaFuncSetAttribute(w8_stream_kernel<kMode, kNT, kTiled>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr_set[dev] = true;
  }
  w8_stream_kernel<kMode, kNT, kTiled><<<grid, kStThreads, smem, stream>>>(
      wa, wb, static_cast<const __nv_bfloat16*>(x), ldx, a);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

template <int kMode, bool kTiled>
int launch_stream_tiled(int nt, dim3 grid, const int8_t* wa, const int8_t* wb, const void* x, int64_t ldx,
                        const StreamArgs& a, cudaStream_t stream) {
  switch (nt) {
    case 8:
      return launch_stream_nt<kMode, 8, kTiled>(grid, wa, wb, x, ldx, a, stream);
    case 16:
      return launch_stream_nt<kMode, 16, kTiled>(grid, wa, wb, x, ldx, a, stream);
    default:
      return launch_stream_nt<kMode, 32, kTiled>(grid, wa, wb, x, ldx, a, stream);
  }
}

template <int kMode>
int launch_stream_mode(int nt, dim3 grid, const int8_t* wa, const int8_t* wb, const void* x,
                       int64_t ldx, const StreamArgs& a, cudaStream_t stream) {
  if (a.w_tiled) return launch_stream_tiled<kMode, true>(nt, grid, wa, wb, x, ldx, a, stream);
  return launch_stream_tiled<kMode, false>(nt, grid, wa, wb, x, ldx, a, stream);
}

}  // namespace

// Work split: ks warps per CTA and kz CTAs share a feature tile's K.  The
// estimate per (ks, kz): CTAs over the resident CTA slots times (the steps
// of a warp + kStCtaSteps of fixed cost: pipeline fill, setup), plus one
// CTA's steps for the last wave; the cheapest with >= 2 steps per warp.
StreamPlan stream_plan(int mode, int nt, bool grouped, bool active_list, int64_t groups,
                       int64_t dense_rows, int64_t routed_rows, int64_t N_out, int64_t K, int kz_max) {
  (void)active_list;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
  const int64_t zc = grouped ? 1 : std::max<int64_t>(1, (dense_rows + nt - 1) / nt);
  const int64_t ftiles = (N_out + 15) / 16;
  const int64_t nsteps = (K + kStStepK - 1) / kStStepK;
  const int64_t active = grouped ? std::max<int64_t>(1, std::min<int64_t>(groups, routed_rows)) : 1;
  const int64_t resident =
      static_cast<int64_t>(num_sms(dev)) * (stream_smem_bytes(epi_is_pair(mode), nt) <= 113 * 1024 ? 2 : 1);
  const int kz_cap = (mode == EPI_COMBINE_F32 || mode == EPI_PLAIN_F32) ? std::max(1, kz_max) : 1;
  StreamPlan best_plan{1, 1};
  double best = 1e300;
  for (int kz = 1; kz <= kz_cap; kz *= 2) {
    for (int k2 = 1; k2 <= kStWarps; k2 *= 2) {
      if ((k2 > 1 || kz > 1) && nsteps / (k2 * kz) < 2) break;
      const int64_t ctas = active * zc * kz * ((ftiles + (kStWarps / k2) - 1) / (kStWarps / k2));
      const double steps = static_cast<double>(nsteps) / (k2 * kz);
      const double cost =
          static_cast<double>(ctas) / static_cast<double>(resident) * (steps + kStCtaSteps) + steps;
      if (cost < best) {
        best = cost;
        best_plan = {k2, kz};
      }
    }
  }
  return best_plan;
}

int launch_gemm_stream(int mode, const int8_t* wa, const int8_t* wb, int64_t groups,
                       int64_t N_out, int64_t K, const void* x, int64_t ldx, int64_t routed_rows,
                       int nt, const StreamArgs& args_in, cudaStream_t stream) {
  const bool pair = epi_is_pair(mode);
  KW8_REQUIRE(K > 0 && K % 16 == 0 && K < (1ll << 31), KW8_ERR_UNSUPPORTED,
              "K=%lld must be a positive multiple of 16", (long long)K);
  KW8_REQUIRE(ldx % 8 == 0 && ldx >= K, KW8_ERR_UNSUPPORTED, "token row pitch %lld invalid",
              (long long)ldx);
  KW8_REQUIRE(N_out > 0 && N_out < (1ll << 31) && groups > 0 && groups <= 65535,
              KW8_ERR_UNSUPPORTED, "shape out of range (N_out=%lld, groups=%lld)",
              (long long)N_out, (long long)groups);
  KW8_REQUIRE(nt == 8 || nt == 16 || nt == 32, KW8_ERR_INVALID_ARG, "token tile %d invalid", nt);
  KW8_REQUIRE(!pair || wb != nullptr, KW8_ERR_INVALID_ARG, "paired GEMM needs two weights");
  KW8_REQUIRE((reinterpret_cast<uintptr_t>(wa) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(wb) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(x) & 15) == 0,
              KW8_ERR_UNSUPPORTED, "operands must be 16-byte aligned");
  KW8_REQUIRE(args_in.group_offsets != nullptr || groups == 1, KW8_ERR_INVALID_ARG,
              "dense mode has one group");
  StreamArgs a = args_in;
  a.K = static_cast<int>(K);
  a.N_out = static_cast<int>(N_out);
  if (a.w_tiled) {
    a.tile_ftiles = static_cast<int>(tiled_ftiles(N_out));
    a.tile_steps = static_cast<int>(tiled_steps(K));
  }
  if (a.group_offsets == nullptr && a.dense_rows <= 0) return KW8_OK;

  const StreamPlan plan = stream_plan(mode, nt, a.group_offsets != nullptr, a.active_groups != nullptr,
                                      groups, a.dense_rows, routed_rows, N_out, K, a.kz_max);
  KW8_REQUIRE(plan.kz == 1 || mode == EPI_COMBINE_F32 || (mode == EPI_PLAIN_F32 && a.split_stride > 0),
              KW8_ERR_INVALID_ARG, "a K split over CTAs needs fp32 partials");
  a.ks = plan.ks;
  a.kz = plan.kz;
  // Dense rows are split over grid z; a group's rows are looped over.
  const int64_t zc =
      a.group_offsets == nullptr ? std::min<int64_t>((a.dense_rows + nt - 1) / nt, 65535) : 1;
  KW8_REQUIRE(zc * plan.kz <= 65535, KW8_ERR_UNSUPPORTED, "too many row passes");
  const int64_t ftiles = (N_out + 15) / 16;
  const int64_t fblocks = (ftiles + (kStWarps / plan.ks) - 1) / (kStWarps / plan.ks);
  KW8_REQUIRE(fblocks < (1ll << 31), KW8_ERR_UNSUPPORTED, "too many feature blocks");
  // With an active-group list at most min(groups, routed rows) groups hold rows.
  const int64_t grid_y = a.active_groups != nullptr
                             ? std::max<int64_t>(1, std::min<int64_t>(groups, routed_rows))
                             : groups;
  const dim3 grid(static_cast<unsigned>(fblocks), static_cast<unsigned>(grid_y),
                  static_cast<unsigned>(zc * plan.kz));
  switch (mode) {
    case EPI_PAIR_GELU:
      return launch_stream_mode<EPI_PAIR_GELU>(nt, grid, wa, wb, x, ldx, a, stream);
    case EPI_PAIR_SILU:
      return launch_stream_mode<EPI_PAIR_SILU>(nt, grid, wa, wb, x, ldx, a, stream);
    case EPI_PLAIN_BF16:
      return launch_stream_mode<EPI_PLAIN_BF16>(nt, grid, wa, wb, x, ldx, a, stream);
    case EPI_PLAIN_F32:
      return launch_stream_mode<EPI_PLAIN_F32>(nt, grid, wa, wb, x, ldx, a, stream);
    case EPI_COMBINE_F32:
      KW8_REQUIRE(a.row_token && a.row_weight, KW8_ERR_INVALID_ARG, "combine needs row maps");
      return launch_stream_mode<EPI_COMBINE_F32>(nt, grid, wa, wb, x, ldx, a, stream);
    default:
      return fail(KW8_ERR_INVALID_ARG, "unknown epilogue mode %d", mode);
  }
}

}  // namespace kw8
