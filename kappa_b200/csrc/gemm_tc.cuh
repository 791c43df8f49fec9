// Grouped W8A16 GEMM on the 5th-generation tensor core (tcgen05, sm_100a).
//
//   out[row][f] = epilogue( scale[f] * Σ_k W[g][f][k] * X[row][k] )
//
// for every row of every group g (an expert, or the single group of a dense
// layer).  W is int8 K-major ([groups][N_out][K]); X is bf16 [rows][K].
//
// A CTA (one per SM, persistent over tiles) runs one pipeline of stages of
// 128 k.  On sm_100a one thread needs ~150 cycles to issue a TMA load and
// ~165 to pass an mbarrier wait, so every per-stage duty is split so that no
// thread's share exceeds the ~512 tensor-core cycles of a stage's 8 MMAs.
// Warps (20 in all):
//   warps 0, 2, 3  TMA producers of stage s (each arms full[s] with its own
//                  bytes): warp 0 the int8 weight tile (128 rows x 128 k,
//                  128 B swizzle), warps 2 and 3 the bf16 token tile's two
//                  64-k halves (nt rows x 128 B, 128 B swizzle).
//   warp 1         MMA issuer (one thread; the warp also allocates TMEM):
//                  per stage 8 x tcgen05.mma kind::f16, M=128 (weight rows),
//                  N=rows of the tile rounded to 16, K=16, A read from TMEM,
//                  B from shared memory, fp32 accumulator in TMEM; it waits
//                  only for aready[s] (the converters saw full[s] first);
//                  tcgen05.commit frees the stage (empty[s]) and, after the
//                  last k tile, hands the accumulator to the epilogue.
//   warps 4..11    converters: warp w owns TMEM lanes 32(w%4)..+31 and one
//                  64-k half of the stage; each thread widens its 64 weights
//                  from int8 to bf16 (exact, two instructions per element)
//                  into the stage's TMEM A slot (tcgen05.st).
//   warps 12..19   epilogue: two warps per lane quarter, alternate 32-column
//                  chunks: read the accumulator (tcgen05.ld), apply the
//                  per-channel scale and the activation, store.
// TMEM (512 columns) holds two accumulators of acc_cols columns (tiles of
// up to 160 tokens; one accumulator above that) followed by one 64-column
// A slot per stage (tc_plan), so the epilogue of one tile overlaps the
// MMAs of the next.
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

#include <atomic>

#include "common.cuh"
#include "pack.cuh"

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
  int nt;         // token rows per tile (multiple of 16, <= kTcMaxNT)
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
  // Weights pre-packed in the tiled layout (kw8_pack_weight) instead of
  // K-major rows: tile_steps 1 KB blocks per 16-row feature tile.
  int a_tiled;
  int tile_steps;
  int tile_ftiles;  // feature tiles per group
  // Split K (EPI_PLAIN_F32 only): each tile's k tiles are cut into
  // k_splits near-equal ranges run by different CTAs; range s writes its
  // partial sums to out + s * split_stride floats (0 or 1: no split).
  int k_splits;
  int64_t split_stride;
  // Pipeline plan (tc_plan), filled in by the launcher.
  int stages, stage_bytes, acc_cols, nbuf;
};

constexpr int kTcMaxStages = 8;                    // pipeline depth limit (barrier arrays)
constexpr int kTcMinDoubleBufferStages = 3;        // fewer stages: one accumulator instead
constexpr int kTcBK = 128;                         // k per stage
constexpr int kTcBHalfK = 64;                      // k per token TMA box (128 B rows)
constexpr int kTcARows = 128;                      // weight rows per tile (M)
constexpr int kTcATileBytes = kTcARows * kTcBK;    // 16 KB int8
constexpr int kTcASlotCols = kTcBK / 2;            // TMEM columns of one stage's bf16 A
constexpr int kTcMaxNT = 256;                      // MMA N limit
constexpr int kTcMaxDoubleBufferNT = 160;          // widest tile with two accumulators
constexpr int kTcDynSmemMax = 232448 - 1024;       // opt-in dynamic smem minus static
constexpr int kTcThreads = 640;                    // 20 warps
constexpr int kTcFirstConvWarp = 4;
constexpr int kTcConvWarps = 8;                    // 2 per TMEM lane quarter (k halves)
constexpr int kTcProducers = 3;                    // warps 0, 2, 3
constexpr int kTcFirstEpiWarp = 12;
constexpr int kTcEpiWarps = 8;                     // 2 per TMEM lane quarter
constexpr uint32_t kTcTmemCols = 512;

// Pipeline plan of one launch, from the token tile nt: accumulator buffers
// of acc_cols TMEM columns (nbuf of them) followed by `stages` A slots of
// 64 columns within the 512 columns; `stages` shared-memory stages of
// stage_bytes (16 KB int8 weights + two 64-k halves of nt x 128 B tokens).
// Two accumulators when that still leaves kTcMinDoubleBufferStages stages.
struct TcPlan {
  int acc_cols, nbuf, stages, stage_bytes, smem_bytes;
};

inline TcPlan tc_plan(int nt) {
  TcPlan pl;
  pl.acc_cols = (nt + 31) & ~31;
  pl.stage_bytes = kTcATileBytes + nt * kTcBK * 2;
  const int smem_stages = (kTcDynSmemMax - 1024) / pl.stage_bytes;
  for (pl.nbuf = 2; pl.nbuf >= 1; --pl.nbuf) {
    const int tmem_stages = (static_cast<int>(kTcTmemCols) - pl.nbuf * pl.acc_cols) / kTcASlotCols;
    pl.stages = std::min(kTcMaxStages, std::min(tmem_stages, smem_stages));
    if (pl.nbuf == 1 || pl.stages >= kTcMinDoubleBufferStages) break;
  }
  pl.smem_bytes = pl.stages * pl.stage_bytes + 1024;  // + 1 KB alignment slack
  return pl;
}

// Largest k_splits <= want for k_tiles k tiles with every range non-empty.
inline int valid_k_splits(int want, int64_t k_tiles) {
  int s = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, k_tiles)));
  while (s > 1 && (s - 1) * ((k_tiles + s - 1) / s) >= k_tiles) --s;
  return s;
}

// out[i] = sum over s < splits of part[s * stride + i] (in that order), as
// fp32 or bf16; n a multiple of 4.
int launch_reduce_splits(const float* part, int splits, int64_t stride, int64_t n, void* out,
                         bool out_bf16, cudaStream_t stream);

// CTA-pair kernel (gemm_tc2.cu): whether a launch takes it (force: 0
// automatic, 1 never, 2 whenever the tile allows), and its launcher.
inline std::atomic<int> g_opt_tc_pair{0};
bool gemm_tc_pair_ok(int mode, int64_t N_out, int nt, int force);
int launch_gemm_tc2(int mode, const int8_t* wa, const int8_t* wb, int64_t groups, int64_t N_out, int64_t K,
                    const void* x, int64_t x_rows, int64_t ldx, const GemmArgs& args_in, int64_t max_entries,
                    cudaStream_t stream);

int launch_gemm_tc(int mode, const int8_t* wa, const int8_t* wb, int64_t groups,
                   int64_t N_out, int64_t K, const void* x, int64_t x_rows,
                   int64_t ldx, const GemmArgs& args_in, cudaStream_t stream);

}  // namespace kw8
