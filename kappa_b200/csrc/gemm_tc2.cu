// Grouped W8A16 GEMM over CTA pairs: tcgen05.mma.cta_group::2 (M = 256).
//
// Same product and epilogues as w8_gemm_tc_kernel (gemm_tc.cu); what
// changes is how a tile is fed.  In the one-CTA kernel every 128-k stage
// moves ~112 KB through one SM's shared memory (TMA writes of the 16 KB
// weight tile and the nt x 256 B token tile, the tensor core's read of the
// token tile, the converters' read of the weights); at 128 B per cycle that
// takes longer than the stage's eight MMAs, so the tensor core waits on
// shared memory (measured with per-stage timestamps: ~900 cycles to issue a
// stage's MMAs against ~640 of MMA work at nt = 160).  Here two CTAs of a
// cluster, on two SMs, compute one 256 x nt tile: each widens its own 128
// weight rows into its own TMEM (the A operand) and loads only half of the
// token tile (the B operand: each CTA's shared memory holds nt/2 rows at
// the same address; the pair's tensor cores read both halves), so the
// token traffic per SM halves and the stage fits its MMA time.
//
// Roles per CTA (20 warps, as in the one-CTA kernel):
//   warp 0      TMA producer of the weight ring (a_stages x 16 KB int8; a
//               tile is free once the converters have read it, so this
//               ring runs far ahead and covers HBM latency);
//   warps 2, 3  TMA producers of the token ring (b_stages x two 64-k halves
//               of nt/2 rows); a token stage is tied to the TMEM A slot of
//               the same index and is free once its MMAs completed;
//   warp 1      CTA 0: the MMA issuer for the pair (8 x tcgen05.mma
//               cta_group::2 per stage, then tcgen05.commit multicast to
//               both CTAs' `empty` barrier); both CTAs: TMEM allocation;
//   warps 4..11 converters: widen the CTA's weight rows int8 -> bf16 into
//               its TMEM A slot, then arrive on CTA 0's `aready` barrier
//               (so CTA 0 learns that both CTAs' slots and token halves are
//               ready);
//   warps 12..19 epilogue of the CTA's 128 output rows (its TMEM
//               accumulator), then arrive on CTA 0's `acc_empty`.
// Every wait is time-bounded like the one-CTA kernel's; both CTAs end with
// a cluster barrier after the MMA issuer's drain, so neither leaves while
// the other's MMAs may still read its memory.
#include "gemm_tc.cuh"

namespace kw8 {

namespace {

struct PairPlan {
  int acc_cols, nbuf, a_stages, b_stages, b_stage_bytes, smem_bytes;
};

// Token tile nt (a multiple of 32): accumulators of acc_cols TMEM columns
// (two while that leaves 3 A slots), b_stages token stages (one per TMEM A
// slot) of nt/2 x 256 B, and as many 16 KB weight stages as shared memory
// holds (at least b_stages, at most kTcMaxStages).
inline PairPlan pair_plan(int nt) {
  PairPlan pl;
  pl.acc_cols = (nt + 31) & ~31;
  pl.b_stage_bytes = (nt / 2) * kTcBK * 2;
  const int budget = kTcDynSmemMax - 1024;  // 1 KB alignment slack
  for (pl.nbuf = 2; pl.nbuf >= 1; --pl.nbuf) {
    const int slots = (static_cast<int>(kTcTmemCols) - pl.nbuf * pl.acc_cols) / kTcASlotCols;
    pl.b_stages = std::min(kTcMaxStages, slots);
    pl.a_stages = 0;
    for (; pl.b_stages >= 2; --pl.b_stages) {
      pl.a_stages = std::min(kTcMaxStages, (budget - pl.b_stages * pl.b_stage_bytes) / kTcATileBytes);
      if (pl.a_stages >= pl.b_stages) break;
    }
    if (pl.nbuf == 1 || pl.b_stages >= kTcMinDoubleBufferStages) break;
  }
  pl.smem_bytes = pl.a_stages * kTcATileBytes + pl.b_stages * pl.b_stage_bytes + 1024;
  return pl;
}

struct PairArgs {
  GemmArgs g;
  int a_stages, b_stages, b_stage_bytes;
};

// MMA N of a tile of `nrows` rows: a multiple of 32 (the pair form's
// granularity), at least 32.
__device__ __forceinline__ int pair_n(int nrows) { return max(32, (nrows + 31) & ~31); }

template <int kMode>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kTcThreads, 1)
    w8_gemm_tc2_kernel(const __grid_constant__ CUtensorMap map_a0,
                       const __grid_constant__ CUtensorMap map_a1,
                       const __grid_constant__ CUtensorMap map_b, const PairArgs pa) {
  constexpr bool kPair = epi_is_pair(kMode);
  const GemmArgs& p = pa.g;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  __shared__ uint64_t full_a[kTcMaxStages];   // weight tile landed (TMA bytes)
  __shared__ uint64_t empty_a[kTcMaxStages];  // weight tile read by this CTA's converters
  __shared__ uint64_t full_b[kTcMaxStages];   // both token halves of this CTA landed
  __shared__ uint64_t aready[kTcMaxStages];   // CTA 0: both CTAs' A slots written (16 warps)
  __shared__ uint64_t empty[kTcMaxStages];    // the stage's MMAs completed (multicast commit)
  __shared__ uint64_t acc_full[2];            // accumulator complete (multicast commit)
  __shared__ uint64_t acc_empty[2];           // CTA 0: both CTAs' epilogues done (16 warps)
  __shared__ uint64_t drain_bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < pa.a_stages; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&empty_a[s], kTcConvWarps);
    }
    for (int s = 0; s < pa.b_stages; ++s) {
      mbar_init(&full_b[s], 2);
      mbar_init(&aready[s], 2 * kTcConvWarps);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kTcEpiWarps);
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
  if (warp == 1) tmem_alloc_pair(&tmem_base_sh, kTcTmemCols);
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised, TMEM allocated
  tc_fence_after();
  volatile int* abort_flag = &abort_sh;

  const int a_stages = pa.a_stages, b_stages = pa.b_stages;
  const int b_stage_bytes = pa.b_stage_bytes;
  const int half_nt = p.nt / 2;
  uint8_t* const smem_a = smem;
  uint8_t* const smem_b = smem + a_stages * kTcATileBytes;
  const uint32_t acc_cols = static_cast<uint32_t>(p.acc_cols);
  const int nbuf = p.nbuf;
  const uint32_t tmem = tmem_base_sh;
  const uint32_t a_col0 = static_cast<uint32_t>(nbuf) * acc_cols;
  // CTA 0's barriers as this CTA addresses them (remote arrivals).
  const uint32_t aready0 = mapa_shared(smem_u32(&aready[0]), 0);
  const uint32_t acc_empty0 = mapa_shared(smem_u32(&acc_empty[0]), 0);

  const int n_entries =
      (p.tiles == nullptr) ? (p.dense_rows + p.nt - 1) / p.nt : *p.num_tiles;
  const int k_tiles = (p.K + kTcBK - 1) / kTcBK;
  const int total_tiles = n_entries * p.m_tiles * (p.k_splits > 1 ? p.k_splits : 1);
  const int pair_id = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  // This CTA's rows of a pair tile: weight rows (128 of the 256) and the
  // output features its TMEM lanes hold.
  const int rows_per_mt = kPair ? 128 : 256;  // features per pair tile

  if (warp == 0 || warp == 2 || warp == 3) {
    if (lane == 0) {
      // ----------------------------------------------- TMA producers ----
      const int part = (warp == 0) ? 0 : warp - 1;  // 0: weights, 1/2: token halves
      const int depth = (part == 0) ? a_stages : b_stages;
      uint64_t* const fullb = (part == 0) ? full_a : full_b;
      uint64_t* const freeb = (part == 0) ? empty_a : empty;
      const uint32_t tx_bytes = (part == 0) ? static_cast<uint32_t>(kTcATileBytes)
                                            : static_cast<uint32_t>(half_nt) * kTcBHalfK * 2;
      const uint32_t b_off = (part == 2) ? static_cast<uint32_t>(half_nt) * kTcBHalfK * 2 : 0u;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, issued_parity = 0;
      bool ok = true;
      for (int t = pair_id; ok && t < total_tiles; t += npairs) {
        const TileInfo ti = decode_tile(p, t, k_tiles);
        const int a_row = ti.group * p.N_out + ti.mt * rows_per_mt + static_cast<int>(crank) * (kPair ? 64 : 128);
        const int b_row = ti.row0 + static_cast<int>(crank) * (pair_n(ti.nrows) / 2);
        for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
          if (!mbar_wait(&freeb[stage], phase ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          // A second token half past K is not loaded (its MMAs are skipped).
          const bool load = part != 2 || kt * kTcBK + kTcBHalfK < p.K;
          if (load)
            mbar_arrive_expect_tx(&fullb[stage], tx_bytes);
          else
            mbar_arrive(&fullb[stage]);
          if (part == 0) {
            uint8_t* dst = smem_a + stage * kTcATileBytes;
            tma_load_2d(dst, &map_a0, &fullb[stage], kt * kTcBK, a_row);
            if (kPair) tma_load_2d(dst + kTcATileBytes / 2, &map_a1, &fullb[stage], kt * kTcBK, a_row);
          } else if (load) {
            tma_load_2d(smem_b + stage * b_stage_bytes + b_off, &map_b, &fullb[stage],
                        kt * kTcBK + (part - 1) * kTcBHalfK, b_row);
          }
          issued_mask |= 1u << stage;
          issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == depth) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Never leave with a TMA write still in flight (time bounded).
      for (int s = 0; s < depth; ++s)
        if (issued_mask & (1u << s)) mbar_wait(&fullb[s], (issued_parity >> s) & 1u, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------- MMA issuer (CTA 0) ----
      int stage = 0, nt_done = 0;
      uint32_t phase = 0, acc_phase = 0;  // acc_phase bit b: phase of buffer b
      bool ok = true;
      const uint32_t b_half = static_cast<uint32_t>(half_nt) * kTcBHalfK * 2;
      for (int t = pair_id; ok && t < total_tiles; t += npairs, ++nt_done) {
        const TileInfo ti = decode_tile(p, t, k_tiles);
        const int ab = nt_done % nbuf;
        const uint32_t idesc = idesc_bf16_f32(256, static_cast<uint32_t>(pair_n(ti.nrows)));
        if (!mbar_wait_cluster(&acc_empty[ab], ((acc_phase >> ab) & 1u) ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(ab) * acc_cols;
        for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
          // Both CTAs' converters arrived: their A slots are written and
          // their token halves have landed.
          if (!mbar_wait_cluster(&aready[stage], phase, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t b_addr = smem_u32(smem_b + stage * b_stage_bytes);
          const uint32_t a_tmem = tmem + a_col0 + stage * kTcASlotCols;
          const int kk_n = min(kTcBK / 16, (p.K - kt * kTcBK) / 16);  // K % 16 == 0
#pragma unroll
          for (int kk = 0; kk < kTcBK / 16; ++kk) {
            if (kk < kk_n) {
              const uint64_t bdesc = smem_desc_kmajor_sw128(b_addr + (kk >> 2) * b_half + (kk & 3) * 32);
              mma_ts_bf16_pair(d_tmem, a_tmem + kk * 8, bdesc, idesc, (kt != ti.kt0 || kk != 0) ? 1u : 0u);
            }
          }
          mma_commit_pair(&empty[stage]);
          if (++stage == b_stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit_pair(&acc_full[ab]);
        acc_phase ^= 1u << ab;
      }
      // Drain: every MMA issued above has completed (and its arrivals on
      // both CTAs' barriers are done) once this arrives.
      mma_commit_pair(&drain_bar);
      mbar_wait(&drain_bar, 0, nullptr);
    } else if (lane == 0) {
      // CTA 1: the pair's last commit also arrives here.
      mbar_wait(&drain_bar, 0, nullptr);
    }
  } else if (warp >= kTcFirstConvWarp && warp < kTcFirstConvWarp + kTcConvWarps) {
    // ------------------------------------------------------ converters ----
    const int q = warp & 3;                         // TMEM lane quarter
    const int kh = (warp - kTcFirstConvWarp) >> 2;  // 64-k half of the stage
    const uint32_t lane_base =
        tmem + (static_cast<uint32_t>(q * 32) << 16) + a_col0 + kh * (kTcASlotCols / 2);
    const int src_row = kPair ? ((lane < 16) ? (q * 16 + lane) : (64 + q * 16 + lane - 16))
                              : (q * 32 + lane);
    const int swz = src_row & 7;  // 128-byte TMA swizzle of this row
    int sa = 0, sb = 0;
    uint32_t pa_ = 0, pb = 0;
    bool ok = true;
    for (int t = pair_id; ok && t < total_tiles; t += npairs) {
      const TileInfo ti = decode_tile(p, t, k_tiles);
      for (int kt = ti.kt0; kt < ti.kt1; ++kt) {
        // Warp-uniform outcomes: the tcgen05.st below needs all 32 lanes.
        if (!__all_sync(0xffffffffu, mbar_wait(&full_a[sa], pa_, abort_flag))) {
          ok = false;
          break;
        }
        const uint8_t* a_src = smem_a + sa * kTcATileBytes + src_row * kTcBK;
        uint32_t v[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint4 w = *reinterpret_cast<const uint4*>(a_src + (((kh * 4 + c) ^ swz) << 4));
          i8x4_to_bf16x4(w.x, v[c * 8 + 0], v[c * 8 + 1]);
          i8x4_to_bf16x4(w.y, v[c * 8 + 2], v[c * 8 + 3]);
          i8x4_to_bf16x4(w.z, v[c * 8 + 4], v[c * 8 + 5]);
          i8x4_to_bf16x4(w.w, v[c * 8 + 6], v[c * 8 + 7]);
        }
        // The weight tile is in registers: hand it back to the producer.
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_a[sa]);
        if (++sa == a_stages) {
          sa = 0;
          pa_ ^= 1u;
        }
        // The A slot is free once the MMAs of its previous stage completed.
        if (!__all_sync(0xffffffffu, mbar_wait(&empty[sb], pb ^ 1u, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        KW8_TMEM_ST_X32(lane_base + sb * kTcASlotCols, v);
        tmem_wait_st();
        tc_fence_before();
        if (!__all_sync(0xffffffffu, mbar_wait(&full_b[sb], pb, abort_flag))) {
          ok = false;
          break;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(aready0 + 8u * static_cast<uint32_t>(sb));
        if (++sb == b_stages) {
          sb = 0;
          pb ^= 1u;
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
    for (int t = pair_id; t < total_tiles; t += npairs, ++nt_done) {
      const TileInfo ti = decode_tile(p, t, k_tiles);
      const int ab = nt_done % nbuf;
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[ab], (acc_phase >> ab) & 1u, abort_flag))) break;
      tc_fence_after();
      const int fbase = ti.mt * rows_per_mt + static_cast<int>(crank) * (kPair ? 64 : 128);
      epilogue_tile<kMode>(p, ti, lane_base + static_cast<uint32_t>(ab) * acc_cols, q, lane, ch,
                           kTcEpiWarps / 4, fbase);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8u * static_cast<uint32_t>(ab));
      acc_phase ^= 1u << ab;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the pair's MMAs are done with both CTAs' memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base_sh, kTcTmemCols);
  }
}

template <int kMode>
int launch_pair_mode(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b, const PairArgs& args,
                     int max_pairs, int smem_bytes, cudaStream_t stream) {
  static bool attr_set[64] = {false};
  static int active_pairs[64][2] = {};  // [dev] -> (smem bytes, co-resident clusters)
  int dev = 0;
  KW8_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) dev = 0;
  if (!attr_set[dev]) {
    KW8_CUDA_TRY(cudaFuncSetAttribute(w8_gemm_tc2_kernel<kMode>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      kTcDynSmemMax));
    attr_set[dev] = true;
  }
  // A persistent grid of as many CTA pairs as can be resident at once (a
  // pair needs two SMs of one GPC).
  if (active_pairs[dev][0] != smem_bytes) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 74, 1, 1);
    cfg.blockDim = dim3(kTcThreads, 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem_bytes);
    int n = 0;
    KW8_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, w8_gemm_tc2_kernel<kMode>, &cfg));
    KW8_REQUIRE(n >= 1, KW8_ERR_UNSUPPORTED, "no CTA pair fits an SM pair");
    active_pairs[dev][0] = smem_bytes;
    active_pairs[dev][1] = n;
  }
  const int pairs = std::max(1, std::min(max_pairs, active_pairs[dev][1]));
  w8_gemm_tc2_kernel<kMode><<<2 * pairs, kTcThreads, smem_bytes, stream>>>(a0, a1, b, args);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

}  // namespace

// Opt-in (force == 2): measured on the Qwen3-30B-A3B expert GEMMs (T = 4096)
// the pair kernel takes 667-809 us against the one-CTA kernel's 415 us over
// token tiles 128-256 (the one-CTA kernel runs at the issue rate of its MMA
// thread, ~160 cycles per tcgen05.mma, at nt = 160; the pair's hand-off
// between the two CTAs' converters and the MMA issuer costs more than the
// halved token traffic saves).  So the automatic choice is the one-CTA
// kernel.
bool gemm_tc_pair_ok(int mode, int64_t N_out, int nt, int force) {
  (void)mode;
  (void)N_out;
  if (force != 2) return false;
  const int nt2 = (nt + 31) & ~31;
  return nt2 >= 32 && nt2 <= kTcMaxNT;
}

// The pair kernel's share of launch_gemm_tc (shapes and alignment checked
// there): token tile rounded up to a multiple of 32, tensor maps with
// 128-row weight boxes (64 + 64 in paired mode) and nt/2-row token boxes.
int launch_gemm_tc2(int mode, const int8_t* wa, const int8_t* wb, int64_t groups, int64_t N_out, int64_t K,
                    const void* x, int64_t x_rows, int64_t ldx, const GemmArgs& args_in, int64_t max_entries,
                    cudaStream_t stream) {
  const bool pair = epi_is_pair(mode);
  PairArgs pa;
  pa.g = args_in;
  pa.g.nt = (args_in.nt + 31) & ~31;
  const PairPlan pl = pair_plan(pa.g.nt);
  KW8_REQUIRE(pl.b_stages >= 2 && pl.b_stages <= kTcMaxStages && pl.a_stages >= pl.b_stages &&
                  pl.a_stages <= kTcMaxStages &&
                  pl.nbuf * pl.acc_cols + pl.b_stages * kTcASlotCols <= static_cast<int>(kTcTmemCols) &&
                  pl.smem_bytes <= kTcDynSmemMax,
              KW8_ERR_INVALID_ARG, "no pair pipeline plan for token tile %d", pa.g.nt);
  pa.g.acc_cols = pl.acc_cols;
  pa.g.nbuf = pl.nbuf;
  pa.a_stages = pl.a_stages;
  pa.b_stages = pl.b_stages;
  pa.b_stage_bytes = pl.b_stage_bytes;
  const int feats = pair ? 128 : 256;  // output features of a pair tile
  pa.g.m_tiles = static_cast<int>((N_out + feats - 1) / feats);

  CUtensorMap map_a0, map_a1, map_b;
  const uint32_t a_box_rows = pair ? 64 : 128;
  int rc = make_tmap_2d(&map_a0, wa, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, static_cast<uint64_t>(groups * N_out),
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
  rc = make_tmap_2d(&map_b, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, static_cast<uint64_t>(x_rows),
                    static_cast<uint64_t>(K), static_cast<uint64_t>(ldx) * 2, kTcBHalfK,
                    static_cast<uint32_t>(pa.g.nt / 2), CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (pa.g.tiles == nullptr) max_entries = (pa.g.dense_rows + pa.g.nt - 1) / pa.g.nt;
  const int64_t max_pairs = max_entries * pa.g.m_tiles * (pa.g.k_splits > 1 ? pa.g.k_splits : 1);
  if (max_pairs <= 0) return KW8_OK;
  const int mp = static_cast<int>(std::min<int64_t>(max_pairs, 1 << 20));
  switch (mode) {
    case EPI_PAIR_GELU:
      return launch_pair_mode<EPI_PAIR_GELU>(map_a0, map_a1, map_b, pa, mp, pl.smem_bytes, stream);
    case EPI_PAIR_SILU:
      return launch_pair_mode<EPI_PAIR_SILU>(map_a0, map_a1, map_b, pa, mp, pl.smem_bytes, stream);
    case EPI_PLAIN_BF16:
      return launch_pair_mode<EPI_PLAIN_BF16>(map_a0, map_a1, map_b, pa, mp, pl.smem_bytes, stream);
    case EPI_PLAIN_F32:
      return launch_pair_mode<EPI_PLAIN_F32>(map_a0, map_a1, map_b, pa, mp, pl.smem_bytes, stream);
    case EPI_COMBINE_F32:
      return launch_pair_mode<EPI_COMBINE_F32>(map_a0, map_a1, map_b, pa, mp, pl.smem_bytes, stream);
    default:
      return fail(KW8_ERR_INVALID_ARG, "unknown epilogue mode %d", mode);
  }
}

}  // namespace kw8
