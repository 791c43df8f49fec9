// Grouped W8A16 GEMM on the 5th-generation tensor core (tcgen05, sm_100a).
//
//   out[row][f] = epilogue( scale[f] * Σ_k W[g][f][k] * X[row][k] )
//
// for every row of every group g (an expert, or the single group of a dense
// layer).  W is int8 K-major ([groups][N_out][K]); X is bf16 [rows][K].
//
// A CTA (one per SM, persistent over tiles) runs two independent pipelines
// ("rings"), each with its own shared-memory stages, half of the 512 TMEM
// columns, its own barriers and every other tile of the CTA's share.  One
// thread can issue a tcgen05.mma only about every 100 cycles, so a single
// issuer keeps the tensor core busy only for tiles of ~200+ tokens; two
// issuers working on 128-token tiles keep it ~90% busy, and while one
// ring drains its accumulator the other still feeds the tensor core.
// Warps of ring r (20 warps in all):
//   warp r         TMA producer: int8 weight tile (128 rows x 64 k, 64 B
//                  swizzle) and bf16 token tile (nt rows x 64 k, 128 B
//                  swizzle) per stage, completion on full[s].
//   warp 2+r       MMA issuer (one thread; warp 2 also allocates TMEM): per
//                  stage 4 x tcgen05.mma kind::f16, M=128 (weight rows),
//                  N=rows of the tile rounded to 16, K=16, A read from TMEM,
//                  B from shared memory, fp32 accumulator in TMEM;
//                  tcgen05.commit frees the stage (empty[s]) and, after the
//                  last k tile, hands the accumulator to the epilogue.
//   warps 4+4r..7+4r   converters: warp w owns TMEM lanes 32(w%4)..+31; each
//                  thread widens its weight row of the stage from int8 to
//                  bf16 (exact) into the stage's TMEM A slot (tcgen05.st).
//   warps 12+4r..15+4r epilogue: read the accumulator (tcgen05.ld), apply
//                  the per-channel scale and the activation, store.
// Each ring's 256 TMEM columns hold its accumulator(s) followed by one
// 32-column A slot per stage (tc_plan); tiles of up to 64 tokens get two
// accumulators per ring.
// Putting the widened weights in TMEM (the "A from TMEM" MMA form) keeps
// the shared-memory traffic per stage at one int8 read plus the tensor
// core's read of the token tile; a bf16 copy of the weights never touches
// shared or global memory.
//
// Paired mode (gate/up of a gated FFN): the 128 weight rows of a tile are
// 64 gate rows and the same 64 up rows.  The converters place gate feature
// f at TMEM lane 32q + (f mod 16) and its up row at lane 32q + 16 + (f mod
// 16), so the epilogue pairs gate and up with one warp shuffle.
#pragma once

#include "common.cuh"

namespace kw8 {

enum EpiMode : int {
  EPI_PAIR_GELU = 0,   // h = gelu_tanh(g) * u, bf16 out, 64 features per tile
  EPI_PAIR_SILU = 1,   // h = silu(g) * u, bf16 out, 64 features per tile
  EPI_PLAIN_BF16 = 2,  // y = acc * s, bf16 out, 128 features per tile
  EPI_PLAIN_F32 = 3,   // y = acc * s, fp32 out, 128 features per tile
  // MoE down projection with the combine fused in: for sorted row p,
  // out[row_token[p]][f] += row_weight[p] * acc * s (fp32 red.add into an
  // L2-resident [T][D] buffer), 128 features per tile.
  EPI_COMBINE_F32 = 4,
};

__host__ __device__ constexpr bool epi_is_pair(int m) {
  return m == EPI_PAIR_GELU || m == EPI_PAIR_SILU;
}

// One work unit of the tile table: rows [row0, row0 + nrows) of group `group`.
// Built on the device from the group offsets (see build_tiles_kernel).
struct TileEntry {
  int group;
  int row0;
  int nrows;
  int pad;
};

struct GemmArgs {
  int K;          // contraction length (multiple of 16)
  int N_out;      // output features per group
  int m_tiles;    // feature tiles per group
  int nt;         // token rows per tile (multiple of 16, <= 256)
  // Tile source: a device table (grouped) or a dense row range.
  const TileEntry* tiles;  // nullptr => dense mode
  const int* num_tiles;    // device count of table entries
  int dense_rows;          // dense mode: rows of the single group
  // Scales (gate/plain = a, up = b).
  const void* scale_a;
  const void* scale_b;
  int scale_a_dtype, scale_b_dtype;
  int scale_a_pc, scale_b_pc;
  // Output [rows][ld_out] ([tokens][ld_out] for EPI_COMBINE_F32).
  void* out;
  int64_t ld_out;
  // EPI_COMBINE_F32 only: token and routing weight of every sorted row.
  const int32_t* row_token;
  const float* row_weight;
  // Pipeline plan (tc_plan), filled in by the launcher.
  int stages, stage_bytes, acc_cols, nbuf;
};

constexpr int kTcRings = 2;
constexpr int kTcMaxStages = 8;                    // pipeline depth limit (barrier arrays)
constexpr int kTcMinDoubleBufferStages = 3;        // fewer stages: one accumulator instead
constexpr int kTcBK = 64;                          // k per stage
constexpr int kTcARows = 128;                      // weight rows per tile (M)
constexpr int kTcATileBytes = kTcARows * kTcBK;    // 8 KB int8
constexpr int kTcMaxNT = 192;                      // one accumulator + 2 A slots per ring
constexpr int kTcDynSmemMax = 232448 - 1024;       // opt-in dynamic smem minus static
constexpr int kTcThreads = 640;                    // 20 warps
constexpr int kTcFirstConvWarp = 4;
constexpr int kTcFirstEpiWarp = 12;
constexpr int kTcEpiWarpsPerRing = 4;
constexpr int kTcMaxDoubleBufferNT = 128;          // widest tile the MoE path asks for
constexpr uint32_t kTcTmemCols = 512;              // allocation (both rings)
constexpr uint32_t kTcRingTmemCols = 256;

// Pipeline plan of one launch, from the token tile nt, per ring:
// accumulator buffers of acc_cols TMEM columns (nbuf of them) followed by
// `stages` A slots of 32 columns, within the ring's 256 columns; `stages`
// shared-memory stages of stage_bytes (8 KB int8 weights + nt x 128 B
// tokens).  Two accumulators when that still leaves
// kTcMinDoubleBufferStages stages.
struct TcPlan {
  int acc_cols, nbuf, stages, stage_bytes, ring_bytes, smem_bytes;
};

inline TcPlan tc_plan(int nt) {
  TcPlan pl;
  pl.acc_cols = (nt + 31) & ~31;
  pl.stage_bytes = kTcATileBytes + nt * kTcBK * 2;
  const int smem_stages = ((kTcDynSmemMax - 1024) / kTcRings) / pl.stage_bytes;
  for (pl.nbuf = 2; pl.nbuf >= 1; --pl.nbuf) {
    const int tmem_stages = (static_cast<int>(kTcRingTmemCols) - pl.nbuf * pl.acc_cols) / 32;
    pl.stages = std::min(kTcMaxStages, std::min(tmem_stages, smem_stages));
    if (pl.nbuf == 1 || pl.stages >= kTcMinDoubleBufferStages) break;
  }
  pl.ring_bytes = pl.stages * pl.stage_bytes;  // multiple of 1024
  pl.smem_bytes = kTcRings * pl.ring_bytes + 1024;  // + 1 KB alignment slack
  return pl;
}

int launch_gemm_tc(int mode, const int8_t* wa, const int8_t* wb, int64_t groups,
                   int64_t N_out, int64_t K, const void* x, int64_t x_rows,
                   int64_t ldx, const GemmArgs& args_in, cudaStream_t stream);

}  // namespace kw8
