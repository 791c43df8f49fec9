// tcgen05 grouped W8A16 GEMM: kernel and launcher.  Design notes are in
// gemm_tc.cuh.
#include "gemm_tc.cuh"

namespace kw8 {

namespace {

struct TileInfo {
  int group, row0, nrows, mt;
  int ks, kt0, kt1;  // K split and its k tiles [kt0, kt1)
};

// Work unit t: K split t % k_splits of feature tile mt of table entry e.
__device__ __forceinline__ TileInfo decode_tile(const GemmArgs& p, int t, int k_tiles) {
  TileInfo ti;
  const int nks = p.k_splits > 1 ? p.k_splits : 1;
  ti.ks = t % nks;
  t /= nks;
  const int per = (k_tiles + nks - 1) / nks;
  ti.kt0 = ti.ks * per;
  ti.kt1 = min(k_tiles, ti.kt0 + per);
  const int e = t / p.m_tiles;
  ti.mt = t - e * p.m_tiles;
  if (p.tiles == nullptr) {
    ti.group = 0;
    ti.row0 = e * p.nt;
    ti.nrows = min(p.nt, p.dense_rows - ti.row0);
  } else {
    const TileEntry te = p.tiles[e];
    ti.group = te.group;
    ti.row0 = te.row0;
    ti.nrows = te.nrows;
  }
  return ti;
}

__device__ __forceinline__ float scale_at(const void* s, int dtype, int pc,
                                          int64_t idx) {
  return load_scale(s, dtype, pc ? idx : 0);
}

// 4x4 transpose within each group of four lanes: lane 4g+p holds a[i] =
// M[p][i] on entry and M[i][p] on exit (two xor-shuffle rounds, one shuffle
// per element).
__device__ __forceinline__ void transpose4x4(float (&a)[4], int lane) {
  const bool b0 = (lane & 1) != 0, b1 = (lane & 2) != 0;
#pragma unroll
  for (int k = 0; k < 2; ++k) {  // 2x2 blocks: exchange elements whose bit 0 differs from p's
    const int j = 2 * k + (b0 ? 0 : 1);
    const float send = b0 ? a[2 * k] : a[2 * k + 1];
    const float got = __shfl_xor_sync(0xffffffffu, send, 1);
    if (b0) a[2 * k] = got; else a[2 * k + 1] = got;
    (void)j;
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {  // blocks of 2x2: exchange elements whose bit 1 differs
    const float send = b1 ? a[k] : a[k + 2];
    const float got = __shfl_xor_sync(0xffffffffu, send, 2);
    if (b1) a[k] = got; else a[k + 2] = got;
  }
}

// Epilogue of one tile for one warp: TMEM lane quarter q, 32-column chunks
// c0, c0 + cstep, ... of the accumulator at acc_lane_base.  The tile's 128
// TMEM lanes hold output features fbase.. (64 paired gate/up features, or
// 128 features).
template <int kMode>
__device__ __forceinline__ void epilogue_tile(const GemmArgs& p, const TileInfo& ti,
                                              uint32_t acc_lane_base, int q, int lane,
                                              int c0, int cstep, int fbase_tile) {
  constexpr bool kPair = epi_is_pair(kMode);
  const int nrows = ti.nrows;
  const int nchunks = (nrows + 31) >> 5;
  if constexpr (kPair) {
    const int f = fbase_tile + q * 16 + (lane & 15);
    const bool fvalid = f < p.N_out;
    const int64_t sidx = static_cast<int64_t>(ti.group) * p.N_out + (fvalid ? f : 0);
    const float s = (lane < 16)
                        ? scale_at(p.scale_a, p.scale_a_dtype, p.scale_a_pc, sidx)
                        : scale_at(p.scale_b, p.scale_b_dtype, p.scale_b_pc, sidx);
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
    const bool hi_half = lane >= 16;
    __nv_bfloat16* col = out + static_cast<int64_t>(ti.row0 + (hi_half ? 16 : 0)) * p.ld_out + f;
    for (int c = c0; c < nchunks; c += cstep) {
      uint32_t r[32];
      KW8_TMEM_LD_X32(acc_lane_base + c * 32, r);
      tmem_wait_ld();
      // All shuffles and math first (no divergence inside), stores after.
      __nv_bfloat16 h[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float lo = __uint_as_float(r[j]) * s;       // token c*32 + j
        const float hi = __uint_as_float(r[16 + j]) * s;  // token c*32 + 16 + j
        const float recv = __shfl_xor_sync(0xffffffffu, hi_half ? lo : hi, 16);
        const float g = hi_half ? recv : lo;
        const float u = hi_half ? hi : recv;
        if constexpr (kMode == EPI_PAIR_GELU)
          h[j] = __float2bfloat16_rn(gelu_tanh_f(g) * u);
        else
          h[j] = __float2bfloat16_rn(silu_f(g) * u);
      }
      // Lane rows: c*32 + j (lanes 0-15) or c*32 + 16 + j (lanes 16-31).
      const int left = nrows - c * 32 - (hi_half ? 16 : 0);
      __nv_bfloat16* dst = col + static_cast<int64_t>(c * 32) * p.ld_out;
      if (fvalid) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (j < left) dst[static_cast<int64_t>(j) * p.ld_out] = h[j];
      }
    }
  } else if constexpr (kMode == EPI_COMBINE_F32) {
    const int fbase = fbase_tile + q * 32;
    const int f = fbase + lane;
    const bool fvalid = f < p.N_out;
    const int64_t sidx = static_cast<int64_t>(ti.group) * p.N_out + (fvalid ? f : 0);
    const float s = scale_at(p.scale_a, p.scale_a_dtype, p.scale_a_pc, sidx);
    const int f4 = fbase + (lane & ~3);  // first of the 4 features this lane adds
    const bool f4valid = f4 < p.N_out;   // N_out % 4 == 0 (checked by the launcher)
    float* out = static_cast<float*>(p.out);
    for (int c = c0; c < nchunks; c += cstep) {
      uint32_t r[32];
      KW8_TMEM_LD_X32(acc_lane_base + c * 32, r);
      // Lane l fetches the token and routing weight of row c*32 + l.
      const int my_row = c * 32 + lane;
      const int tok_l = (my_row < nrows) ? p.row_token[ti.row0 + my_row] : 0;
      const float w_l = (my_row < nrows) ? p.row_weight[ti.row0 + my_row] : 0.f;
      tmem_wait_ld();
      // Rows 4b..4b+3 of the chunk; after the transpose lane 4g+pl holds
      // features f4..f4+3 of row 4b+pl, added with one 16-byte atomic.  All
      // shuffles first (no divergence inside), atomics after.
      float4 v[8];
      int tok[8];
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        float a[4] = {__uint_as_float(r[4 * b]) * s, __uint_as_float(r[4 * b + 1]) * s,
                      __uint_as_float(r[4 * b + 2]) * s, __uint_as_float(r[4 * b + 3]) * s};
        transpose4x4(a, lane);
        const int src = 4 * b + (lane & 3);
        tok[b] = __shfl_sync(0xffffffffu, tok_l, src);
        const float wr = __shfl_sync(0xffffffffu, w_l, src);
        v[b] = make_float4(a[0] * wr, a[1] * wr, a[2] * wr, a[3] * wr);
      }
      const int left = nrows - c * 32 - (lane & 3);
      if (f4valid) {
#pragma unroll
        for (int b = 0; b < 8; ++b)
          if (4 * b < left)
            atomicAdd(reinterpret_cast<float4*>(out + static_cast<int64_t>(tok[b]) * p.ld_out + f4),
                      v[b]);
      }
    }
  } else {
    const int f = fbase_tile + q * 32 + lane;
    const bool fvalid = f < p.N_out;
    const int64_t sidx = static_cast<int64_t>(ti.group) * p.N_out + (fvalid ? f : 0);
    const float s = scale_at(p.scale_a, p.scale_a_dtype, p.scale_a_pc, sidx);
    for (int c = c0; c < nchunks; c += cstep) {
      uint32_t r[32];
      KW8_TMEM_LD_X32(acc_lane_base + c * 32, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int tok = c * 32 + j;
        if (fvalid && tok < nrows) {
          const float y = __uint_as_float(r[j]) * s;
          const int64_t o = static_cast<int64_t>(ti.row0 + tok) * p.ld_out + f;
          if constexpr (kMode == EPI_PLAIN_F32)
            static_cast<float*>(p.out)[o + ti.ks * p.split_stride] = y;
          else
            static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(y);
        }
      }
    }
  }
}

template <int kMode>
__global__ void __launch_bounds__(kTcThreads, 1)
    w8_gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a0,
                      const __grid_constant__ CUtensorMap map_a1,
                      const __grid_constant__ CUtensorMap map_b,
                      const GemmArgs p) {
  constexpr bool kPair = epi_is_pair(kMode);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  __shared__ uint64_t full[kTcMaxStages];
  __shared__ uint64_t aready[kTcMaxStages];
  __shared__ uint64_t empty[kTcMaxStages];
  __shared__ uint64_t acc_full[2];
  __shared__ uint64_t acc_empty[2];
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], kTcProducers);
      mbar_init(&aready[s], kTcConvWarps);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kTcEpiWarps);
    }
    mbar_init(&drain_bar, 1);
    abort_sh = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a0);
    if (kPair) tma_prefetch_desc(&map_a1);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) tmem_alloc(&tmem_base_sh, kTcTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  volatile int* abort_flag = &abort_sh;

  // Plan from the launcher (tc_plan).
  const int kStages = p.stages;
  const int stage_bytes = p.stage_bytes;
  const uint32_t acc_cols = static_cast<uint32_t>(p.acc_cols);
  const int nbuf = p.nbuf;
  const uint32_t tmem = tmem_base_sh;
  const uint32_t a_col0 = static_cast<uint32_t>(nbuf) * acc_cols;

  const int n_entries =
      (p.tiles == nullptr) ? (p.dense_rows + p.nt - 1) / p.nt : *p.num_tiles;
  const int k_tiles = (p.K + kTcBK - 1) / kTcBK;
  const int total_tiles = n_entries * p.m_tiles * (p.k_splits > 1 ? p.k_splits : 1);

  if (warp == 0 || warp == 2 || warp == 3) {
    if (lane == 0) {
      // ----------------------------------------------- TMA producers ----
      // Warp 0 loads the weight tile, warps 2 and 3 one 64-k half of the
      // token tile each; each arms full[s] with its own bytes.
      const int part = (warp == 0) ? 0 : warp - 1;  // 0: weights, 1/2: token halves
      const uint32_t tx_bytes = (part == 0)
                                    ? static_cast<uint32_t>(kTcATileBytes)
                                    : static_cast<uint32_t>(p.nt) * kTcBHalfK * 2;
      const uint32_t b_off = kTcATileBytes + (part == 2 ? p.nt * kTcBHalfK * 2 : 0);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total_tiles; t += gridDim.x) {
        const TileInfo ti = decode_tile(p, t, k_tiles);
        const int a_row = ti.group * p.N_out + ti.mt * (kPair ? 64 : 128);
        for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* dst = smem + stage * stage_bytes;
          // A second token half past K is not loaded (its MMAs are skipped).
          const bool load = part != 2 || kt * kTcBK + kTcBHalfK < p.K;
          if (load)
            mbar_arrive_expect_tx(&full[stage], tx_bytes);
          else
            mbar_arrive(&full[stage]);
          if (part == 0) {
            if (p.a_tiled) {
              // One box = the stage's 8 (paired: 4 + 4) feature tiles x 2 steps.
              const int z = ti.group * p.tile_ftiles + ti.mt * (kPair ? 4 : 8);
              tma_load_3d(dst, &map_a0, &full[stage], 0, kt * 8, z);
              if (kPair) tma_load_3d(dst + kTcATileBytes / 2, &map_a1, &full[stage], 0, kt * 8, z);
            } else if (kPair) {
              tma_load_2d(dst, &map_a0, &full[stage], kt * kTcBK, a_row);
              tma_load_2d(dst + kTcATileBytes / 2, &map_a1, &full[stage], kt * kTcBK, a_row);
            } else {
              tma_load_2d(dst, &map_a0, &full[stage], kt * kTcBK, a_row);
            }
          } else if (load) {
            tma_load_2d(dst + b_off, &map_b, &full[stage], kt * kTcBK + (part - 1) * kTcBHalfK,
                        ti.row0);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Never leave the CTA with a TMA write still in flight: wait (time
      // bounded, abort ignored) for the last phase armed on each stage.
      for (int s = 0; s < kStages; ++s)
        if (issued_mask & (1u << s))
          mbar_wait(&full[s], (issued_parity >> s) & 1u, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------- MMA issuer ----
      int stage = 0, nt_done = 0;
      uint32_t phase = 0, acc_phase = 0;  // acc_phase bit b: phase of buffer b
      bool ok = true;
      for (int t = blockIdx.x; ok && t < total_tiles; t += gridDim.x, ++nt_done) {
        const TileInfo ti = decode_tile(p, t, k_tiles);
        const int ab = nt_done % nbuf;
        const uint32_t n_mma = static_cast<uint32_t>(max(16, (ti.nrows + 15) & ~15));
        const uint32_t idesc = idesc_bf16_f32(128, n_mma);
        if (!mbar_wait(&acc_empty[ab], ((acc_phase >> ab) & 1u) ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(ab) * acc_cols;
        for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
          // aready[s] completes after every converter saw full[s], so the
          // token tile of the stage has landed as well.
          if (!mbar_wait(&aready[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_addr = smem_u32(smem + stage * stage_bytes + kTcATileBytes);
          const uint32_t b_half = static_cast<uint32_t>(p.nt) * kTcBHalfK * 2;
          const uint32_t a_tmem = tmem + a_col0 + stage * kTcASlotCols;
          const int kk_n = min(kTcBK / 16, (p.K - kt * kTcBK) / 16);  // K % 16 == 0
#pragma unroll
          for (int kk = 0; kk < kTcBK / 16; ++kk) {
            if (kk < kk_n) {
              const uint64_t bdesc =
                  smem_desc_kmajor_sw128(b_addr + (kk >> 2) * b_half + (kk & 3) * 32);
              mma_ts_bf16(d_tmem, a_tmem + kk * 8, bdesc, idesc, (kt != ti.kt0 || kk != 0) ? 1u : 0u);
            }
          }
          mma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&acc_full[ab]);
        acc_phase ^= 1u << ab;
      }
      // Drain: every MMA issued above has completed once this arrives.
      mma_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, nullptr);
    }
  } else if (warp >= kTcFirstConvWarp && warp < kTcFirstConvWarp + kTcConvWarps) {
    // ------------------------------------------------------ converters ----
    const int q = warp & 3;                               // TMEM lane quarter
    const int kh = (warp - kTcFirstConvWarp) >> 2;        // 64-k half of the stage
    const uint32_t lane_base =
        tmem + (static_cast<uint32_t>(q * 32) << 16) + a_col0 + kh * (kTcASlotCols / 2);
    const int src_row = kPair ? ((lane < 16) ? (q * 16 + lane) : (64 + q * 16 + lane - 16))
                              : (q * 32 + lane);
    const int swz = src_row & 7;  // 128-byte TMA swizzle of this row
    // Offsets of this thread's four 16-byte chunks within a stage: K-major
    // tiles, 128-byte rows swizzled by (row & 7); tiled weights, row r's chunk
    // c of step kh at (r/16) * 2 KB + kh * 1 KB + 512 ((r % 16) / 8) + 16 (8 c + r % 8).
    uint32_t coff[4];
#pragma unroll
    for (int c = 0; c < 4; ++c)
      coff[c] = p.a_tiled ? static_cast<uint32_t>((src_row >> 4) * 2048 + kh * 1024 + ((src_row >> 3) & 1) * 512 +
                                                  (src_row & 7) * 16 + c * 128)
                          : static_cast<uint32_t>(src_row * kTcBK + (((kh * 4 + c) ^ swz) << 4));
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < total_tiles; t += gridDim.x) {
      const TileInfo ti = decode_tile(p, t, k_tiles);
      for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
        // Warp-uniform outcome: the tcgen05.st below needs all 32 lanes.
        if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], phase, abort_flag))) {
          ok = false;
          break;
        }
        const uint8_t* a_stage = smem + stage * stage_bytes;
        uint32_t v[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 w = *reinterpret_cast<const uint4*>(a_stage + coff[c]);
          i8x4_to_bf16x4(w.x, v[c * 8 + 0], v[c * 8 + 1]);
          i8x4_to_bf16x4(w.y, v[c * 8 + 2], v[c * 8 + 3]);
          i8x4_to_bf16x4(w.z, v[c * 8 + 4], v[c * 8 + 5]);
          i8x4_to_bf16x4(w.w, v[c * 8 + 6], v[c * 8 + 7]);
        }
        KW8_TMEM_ST_X32(lane_base + stage * kTcASlotCols, v);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&aready[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp >= kTcFirstEpiWarp) {
    // -------------------------------------------------------- epilogue ----
    const int q = warp & 3;
    const int ch = (warp - kTcFirstEpiWarp) >> 2;  // chunks ch, ch + 2, ...
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    uint32_t acc_phase = 0;
    int nt_done = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x, ++nt_done) {
      const TileInfo ti = decode_tile(p, t, k_tiles);
      const int ab = nt_done % nbuf;
      if (!__all_sync(0xffffffffu,
                      mbar_wait(&acc_full[ab], (acc_phase >> ab) & 1u, abort_flag)))
        break;
      tc_fence_after();
      epilogue_tile<kMode>(p, ti, lane_base + static_cast<uint32_t>(ab) * acc_cols, q, lane, ch,
                           kTcEpiWarps / 4, ti.mt * (kPair ? 64 : 128));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
      acc_phase ^= 1u << ab;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base_sh, kTcTmemCols);
  }
}

int g_num_sms[64] = {0};

int num_sms(int dev) {
  if (dev < 0 || dev >= 64) return 148;
  if (g_num_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_num_sms[dev] = n;
  }
  return g_num_sms[dev];
}

template <int kMode>
int launch_mode(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b,
                const GemmArgs& args, int grid, cudaStream_t stream) {
  static bool attr_set[64] = {false};
  int dev = 0;
  KW8_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    KW8_CUDA_TRY(cudaFuncSetAttribute(w8_gemm_tc_kernel<kMode>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kTcDynSmemMax));
    attr_set[dev] = true;
  }
  const TcPlan pl = tc_plan(args.nt);
  w8_gemm_tc_kernel<kMode><<<grid, kTcThreads, pl.smem_bytes, stream>>>(a0, a1, b, args);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

}  // namespace

namespace {

__global__ void reduce_splits_kernel(const float4* __restrict__ part, int splits, int64_t stride4, int64_t n4,
                                     void* out, int out_bf16) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 a = part[i];
    for (int s = 1; s < splits; ++s) {
      const float4 b = part[s * stride4 + i];
      a.x += b.x;
      a.y += b.y;
      a.z += b.z;
      a.w += b.w;
    }
    if (out_bf16) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y), hi = __floats2bfloat162_rn(a.z, a.w);
      uint2 v;
      v.x = *reinterpret_cast<uint32_t*>(&lo);
      v.y = *reinterpret_cast<uint32_t*>(&hi);
      static_cast<uint2*>(out)[i] = v;
    } else {
      static_cast<float4*>(out)[i] = a;
    }
  }
}

}  // namespace

int launch_reduce_splits(const float* part, int splits, int64_t stride, int64_t n, void* out,
                         bool out_bf16, cudaStream_t stream) {
  KW8_REQUIRE(n % 4 == 0 && stride % 4 == 0 && splits >= 1 &&
                  (reinterpret_cast<uintptr_t>(part) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(out) & (out_bf16 ? 7 : 15)) == 0,
              KW8_ERR_UNSUPPORTED, "split reduction needs 4-element alignment");
  if (n <= 0) return KW8_OK;
  const int64_t n4 = n / 4;
  const int64_t blocks = std::min<int64_t>((n4 + 255) / 256, 148 * 8);
  reduce_splits_kernel<<<static_cast<int>(blocks), 256, 0, stream>>>(
      reinterpret_cast<const float4*>(part), splits, stride / 4, n4, out, out_bf16 ? 1 : 0);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

// Launches the grouped GEMM.  `wa` (and `wb` in paired mode) are int8
// [groups][N_out][K]; x is bf16 [x_rows][ldx].  `args_in` carries the tile
// source, scales and output; the launcher fills in the shape fields.
int launch_gemm_tc(int mode, const int8_t* wa, const int8_t* wb, int64_t groups,
                   int64_t N_out, int64_t K, const void* x, int64_t x_rows,
                   int64_t ldx, const GemmArgs& args_in, cudaStream_t stream) {
  const bool pair = epi_is_pair(mode);
  KW8_REQUIRE(K > 0 && K % 16 == 0, KW8_ERR_UNSUPPORTED, "K=%lld must be a positive multiple of 16",
              (long long)K);
  KW8_REQUIRE(ldx % 8 == 0 && ldx >= K, KW8_ERR_UNSUPPORTED, "token row pitch %lld invalid",
              (long long)ldx);
  KW8_REQUIRE(N_out > 0 && groups > 0 && groups * N_out < (1ll << 31), KW8_ERR_UNSUPPORTED,
              "weight rows out of range");
  KW8_REQUIRE(x_rows > 0 && x_rows < (1ll << 31), KW8_ERR_UNSUPPORTED, "token rows out of range");
  KW8_REQUIRE(args_in.nt >= 16 && args_in.nt <= kTcMaxNT && args_in.nt % 16 == 0,
              KW8_ERR_INVALID_ARG, "token tile %d invalid", args_in.nt);
  KW8_REQUIRE(!pair || wb != nullptr, KW8_ERR_INVALID_ARG, "paired GEMM needs two weights");
  KW8_REQUIRE((reinterpret_cast<uintptr_t>(wa) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(wb) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(x) & 15) == 0,
              KW8_ERR_UNSUPPORTED, "operands must be 16-byte aligned");

  GemmArgs args = args_in;
  args.K = static_cast<int>(K);
  args.N_out = static_cast<int>(N_out);
  if (mode == EPI_COMBINE_F32) {
    KW8_REQUIRE(args.row_token && args.row_weight, KW8_ERR_INVALID_ARG, "combine needs row maps");
    KW8_REQUIRE(N_out % 4 == 0 && args.ld_out % 4 == 0 && (reinterpret_cast<uintptr_t>(args.out) & 15) == 0,
                KW8_ERR_UNSUPPORTED, "fused combine needs D %% 4 == 0 and a 16-byte aligned output");
  }
  if (args.k_splits > 1) {
    const int64_t kt = (K + kTcBK - 1) / kTcBK;
    KW8_REQUIRE(mode == EPI_PLAIN_F32 && args.k_splits == valid_k_splits(args.k_splits, kt) &&
                    args.split_stride > 0,
                KW8_ERR_INVALID_ARG, "split K needs fp32 output, non-empty ranges and a stride");
  }
  if (!args.a_tiled && gemm_tc_pair_ok(mode, N_out, args.nt, g_opt_tc_pair.load())) {
    // Feature tiles of 256 rows over an SM pair (gemm_tc2.cu).
    const int64_t max_entries = args.tiles == nullptr ? 0 : groups + (x_rows + args.nt - 1) / args.nt;
    return launch_gemm_tc2(mode, wa, wb, groups, N_out, K, x, x_rows, ldx, args, max_entries, stream);
  }
  const TcPlan pl = tc_plan(args.nt);
  KW8_REQUIRE(pl.stages >= 2 && pl.stages <= kTcMaxStages &&
                  pl.nbuf * pl.acc_cols + pl.stages * kTcASlotCols <= static_cast<int>(kTcTmemCols) &&
                  pl.smem_bytes <= kTcDynSmemMax,
              KW8_ERR_INVALID_ARG, "no pipeline plan for token tile %d", args.nt);
  args.stages = pl.stages;
  args.stage_bytes = pl.stage_bytes;
  args.acc_cols = pl.acc_cols;
  args.nbuf = pl.nbuf;
  const int rows_per_mtile = pair ? 64 : 128;
  args.m_tiles = static_cast<int>((N_out + rows_per_mtile - 1) / rows_per_mtile);

  CUtensorMap map_a0, map_a1, map_b;
  const uint32_t a_box_rows = pair ? 64 : 128;
  int rc;
  if (args.a_tiled) {
    args.tile_ftiles = static_cast<int>(tiled_ftiles(N_out));
    args.tile_steps = static_cast<int>(tiled_steps(K));
    const uint64_t tile_rows = static_cast<uint64_t>(groups) * args.tile_ftiles;
    rc = make_tmap_tiled(&map_a0, wa, tile_rows, args.tile_steps, a_box_rows / 16);
    if (!rc && pair) rc = make_tmap_tiled(&map_a1, wb, tile_rows, args.tile_steps, a_box_rows / 16);
    if (rc) return rc;
    if (!pair) map_a1 = map_a0;
  } else {
    rc = make_tmap_2d(&map_a0, wa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, static_cast<uint64_t>(groups * N_out),
                      static_cast<uint64_t>(K), static_cast<uint64_t>(K), kTcBK, a_box_rows,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (pair) {
      rc = make_tmap_2d(&map_a1, wb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, static_cast<uint64_t>(groups * N_out),
                        static_cast<uint64_t>(K), static_cast<uint64_t>(K), kTcBK, a_box_rows,
                        CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
    } else {
      map_a1 = map_a0;
    }
  }
  rc = make_tmap_2d(&map_b, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                    static_cast<uint64_t>(x_rows), static_cast<uint64_t>(K),
                    static_cast<uint64_t>(ldx) * 2, kTcBHalfK, static_cast<uint32_t>(args.nt),
                    CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;

  // Upper bound on the work: the table holds at most groups + rows/nt
  // entries; a dense range holds ceil(rows/nt).
  int64_t max_entries = args.tiles == nullptr
                            ? (args.dense_rows + args.nt - 1) / args.nt
                            : groups + (x_rows + args.nt - 1) / args.nt;
  const int64_t k_tiles = (K + kTcBK - 1) / kTcBK;
  if (args.k_splits > 1) {
    KW8_REQUIRE(mode == EPI_PLAIN_F32 && args.k_splits == valid_k_splits(args.k_splits, k_tiles) &&
                    args.split_stride > 0,
                KW8_ERR_INVALID_ARG, "split K needs fp32 output, non-empty ranges and a stride");
  }
  int64_t max_tiles = max_entries * args.m_tiles * (args.k_splits > 1 ? args.k_splits : 1);
  if (max_tiles <= 0) return KW8_OK;
  int dev = 0;
  KW8_CUDA_TRY(cudaGetDevice(&dev));
  const int grid = static_cast<int>(std::min<int64_t>(max_tiles, num_sms(dev)));

  switch (mode) {
    case EPI_PAIR_GELU:
      return launch_mode<EPI_PAIR_GELU>(map_a0, map_a1, map_b, args, grid, stream);
    case EPI_PAIR_SILU:
      return launch_mode<EPI_PAIR_SILU>(map_a0, map_a1, map_b, args, grid, stream);
    case EPI_PLAIN_BF16:
      return launch_mode<EPI_PLAIN_BF16>(map_a0, map_a1, map_b, args, grid, stream);
    case EPI_PLAIN_F32:
      return launch_mode<EPI_PLAIN_F32>(map_a0, map_a1, map_b, args, grid, stream);
    case EPI_COMBINE_F32:
      KW8_REQUIRE(args.row_token && args.row_weight, KW8_ERR_INVALID_ARG, "combine needs row maps");
      KW8_REQUIRE(N_out % 4 == 0 && args.ld_out % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(args.out) & 15) == 0,
                  KW8_ERR_UNSUPPORTED, "fused combine needs D %% 4 == 0 and a 16-byte aligned output");
      return launch_mode<EPI_COMBINE_F32>(map_a0, map_a1, map_b, args, grid, stream);
    default:
      return fail(KW8_ERR_INVALID_ARG, "unknown epilogue mode %d", mode);
  }
}

}  // namespace kw8
