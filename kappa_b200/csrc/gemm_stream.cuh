// Grouped W8A16 weight-streaming GEMM for few token rows per group (decode).
//
//   out[row][f] = epilogue( scale[f] * sum_k W[g][f][k] * X[row][k] )
//
// When a group holds only a few rows the work is bound by int8 weight bytes,
// not by arithmetic: every weight byte is used for at most a few dozen
// multiply-adds.  This kernel streams each weight row once from HBM: every
// lane copies its own 16-byte chunks of weights and token rows into a
// per-warp shared-memory ring (cp.async, a few steps deep), widens int8 to
// bf16 exactly in registers and multiplies on the tensor core with
// mma.sync.m16n8k16 (bf16 in, fp32 accumulate).  A lane reads back only the
// chunks it copied, so its own wait_group is the only synchronisation: no
// mbarriers and no tile table.  A CTA reads its group's row range from the
// group offsets, and token rows are read through an optional row index (the
// permutation's token of each sorted row), so the gather of the routed rows
// is fused into the operand load.  (Measured and dropped: bulk L2
// prefetches of the weight rows, 128-k steps, token rows staged once per
// CTA in shared memory as bf16 or as f16 with f16 weights; all slower.)
//
// A warp owns 16 output features (16 gate + 16 up rows in paired mode) and
// one slice of K; a CTA of 8 warps covers 8/ks feature tiles x ks K slices
// (partial sums of the slices meet in shared memory, added in slice order).
// Within a warp step of 64 k, lane (g, c) = (lane / 4, lane % 4) loads 16
// consecutive k of feature rows g and g + 8 at k0 + 16c and the same 16 k
// of token row g of each 8-row token tile; MMA j (0..3) of the step takes
// k0 + 16c + 4j + {0,1} as its fragment columns 2c, 2c+1 and
// k0 + 16c + 4j + {2,3} as columns 2c+8, 2c+9.  A and B use the same
// assignment, so every k of the step meets its partner exactly once.
#pragma once

#include "gemm_tc.cuh"

namespace kw8 {

struct StreamArgs {
  int K;      // contraction length (multiple of 16)
  int N_out;  // output features per group
  // Row source: group g owns sorted rows [group_offsets[g], group_offsets[g+1]);
  // nullptr => one group of dense_rows rows.
  const int32_t* group_offsets;
  int dense_rows;
  // Optional list of the groups holding rows (active[0] = count, then the
  // groups): grid row y serves group active[1 + y], so empty groups cost no
  // CTAs.  nullptr: grid row y serves group y.
  const int32_t* active_groups;
  // x row of sorted row r: row_index[r] (fused gather), or r when nullptr.
  const int32_t* row_index;
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
  // K split over CTAs: at most kz_max ranges (EPI_COMBINE_F32: any, its
  // atomics add the ranges; EPI_PLAIN_F32: range r writes out + r *
  // split_stride floats, the caller sums them; other modes: 1).
  int kz_max;
  int64_t split_stride;
  // Weights pre-packed in the tiled layout (kw8_pack_weight): tile_steps
  // 1 KB blocks per 16-row feature tile, tile_ftiles tiles per group.
  int w_tiled;
  int tile_steps, tile_ftiles;
  // Filled in by the launcher (stream_plan).
  int ks;  // warps of a CTA splitting its K range (1, 2, 4 or 8)
  int kz;  // CTAs splitting K
};

// Work split of a launch: K ranges over kz CTAs and ks warps per CTA.
struct StreamPlan {
  int ks, kz;
};

// The split launch_gemm_stream uses for these arguments (callers size the
// EPI_PLAIN_F32 partial buffer and decide on the reduction with it).
StreamPlan stream_plan(int mode, int nt, bool grouped, bool active_list, int64_t groups,
                       int64_t dense_rows, int64_t routed_rows, int64_t N_out, int64_t K, int kz_max);

constexpr int kStreamMaxNT = 32;  // token rows per pass of a CTA over its weights

// Token rows per pass for groups of `rows_hint` rows (8, 16 or 32).
inline int stream_nt(double rows_hint) {
  if (rows_hint <= 8.0) return 8;
  if (rows_hint <= 16.0) return 16;
  return 32;
}

// `groups` groups of N_out x K int8 weights (paired mode: `wa` gate, `wb`
// up); x is bf16 [x_rows][ldx].  `nt` is 8, 16 or 32; `routed_rows` (the
// rows of all groups) sizes the grid.
int launch_gemm_stream(int mode, const int8_t* wa, const int8_t* wb, int64_t groups,
                       int64_t N_out, int64_t K, const void* x, int64_t ldx, int64_t routed_rows,
                       int nt, const StreamArgs& args_in, cudaStream_t stream);

}  // namespace kw8
