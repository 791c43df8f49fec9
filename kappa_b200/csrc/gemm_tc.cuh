// Grouped W8A16 GEMM on the 5th-generation tensor core (tcgen05, sm_100a).
//
//   out[row][f] = epilogue( scale[f] * Σ_k W[g][f][k] * X[row][k] )
//
// for every row of every group g (an expert, or the single group of a dense
// layer).  W is int8 K-major ([groups][N_out][K]); X is bf16 [rows][K].
//
// Roles of the 20 warps of a CTA (one CTA per SM, persistent over tiles):
//   warp 0       TMA producer: int8 weight tile (128 rows x 64 k, 64 B
//                swizzle) and bf16 token tile (nt rows x 64 k, 128 B swizzle)
//                per pipeline stage, completion on full[s].
//   warp 1       TMEM allocator and MMA issuer (one thread): per stage,
//                4 x tcgen05.mma kind::f16, M=128 (weight rows), N=rows of
//                the tile rounded to 16, K=16, A read from TMEM, B from
//                shared memory, accumulator in TMEM; tcgen05.commit frees the
//                stage (empty[s]) and, after the last k tile, hands the
//                accumulator to the epilogue (acc_full[b]).
//   warps 4-11   converters, two groups of four that take alternate
//                stages.  Warp w owns TMEM lanes 32(w%4)..+31; each thread
//                widens its weight row of the stage from int8 to bf16
//                (exact) into the stage's TMEM A slot (tcgen05.st), then
//                the warp arrives on a_ready[s].
//   warps 12-19  epilogue, two warps per TMEM lane quarter taking alternate
//                32-column chunks: read the fp32 accumulator (tcgen05.ld),
//                apply the per-channel scale and the activation, store.
// When the token tile is at most 160 columns the accumulator is double
// buffered in TMEM (2 x 160 + 5 A slots x 32 = 480 of 512 columns), so the
// epilogue of one tile runs under the MMAs of the next; wider tiles use one
// accumulator and the MMA waits for the epilogue.
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
};

constexpr int kTcStages = 5;
constexpr int kTcBK = 64;                          // k per stage
constexpr int kTcARows = 128;                      // weight rows per tile (M)
constexpr int kTcATileBytes = kTcARows * kTcBK;    // 8 KB int8
constexpr int kTcMaxNT = 256;
constexpr int kTcBTileBytes = kTcMaxNT * kTcBK * 2;  // 32 KB bf16
constexpr int kTcStageBytes = kTcATileBytes + kTcBTileBytes;
constexpr int kTcSmemBytes = kTcStages * kTcStageBytes + 1024;  // + align slack
constexpr int kTcThreads = 640;
constexpr int kTcConvGroups = 2;        // converter groups (4 warps each)
constexpr int kTcFirstConvWarp = 4;
constexpr int kTcFirstEpiWarp = 12;
constexpr int kTcEpiWarps = 8;          // two per TMEM lane quarter
constexpr int kTcMaxDoubleBufferNT = 160;  // widest tile with two accumulators
static_assert(2 * ((kTcMaxDoubleBufferNT + 31) / 32 * 32) + kTcStages * 32 <= 512,
              "two accumulators and the A slots must fit in 512 TMEM columns");
static_assert(kTcMaxNT + kTcStages * 32 <= 512, "one accumulator and the A slots must fit");
constexpr uint32_t kTcTmemCols = 512;
// TMEM columns: accumulator buffer b at [b * acc_cols, +acc_cols) with
// acc_cols = nt rounded up to 32; A slot s at [nbuf * acc_cols + 32 s, +32).

int launch_gemm_tc(int mode, const int8_t* wa, const int8_t* wb, int64_t groups,
                   int64_t N_out, int64_t K, const void* x, int64_t x_rows,
                   int64_t ldx, const GemmArgs& args_in, cudaStream_t stream);

}  // namespace kw8
