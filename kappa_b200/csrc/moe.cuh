// MoE routing kernels (see moe.cu).
#pragma once

#include "gemm_tc.cuh"

namespace kw8 {

// With zero_rows: also zeroes zero_rows[T][zero_cols] (fp32, zero_cols % 4 == 0).
int launch_topk(const float* logits, int64_t T, int64_t E, int k, int32_t* idx, void* w,
                cudaStream_t stream, float* zero_rows = nullptr, int64_t zero_cols = 0);
// Top-k + softmax, stable permutation (as launch_permute_multi, with the
// active-expert list) and the zeroing of zero_rows[T][zero_cols] in one
// launch, for route_tail_small_ok shapes (decode batches).
constexpr int kTailMaxRows = 256;
inline bool route_tail_small_ok(int64_t T, int64_t E, int k) {
  return T >= 1 && k >= 1 && k <= 32 && k <= E && E <= 256 && T * k <= kTailMaxRows;
}
int launch_route_tail_small(const float* logits, int64_t T, int64_t E, int k, int64_t capacity,
                            int32_t* idx, void* w, int32_t* sorted_token, int32_t* inv_pos,
                            int32_t* group_sizes, int32_t* group_offsets, float* sorted_w,
                            int32_t* active, float* zero_rows, int64_t zero_cols,
                            cudaStream_t stream);
// `w` / `sorted_w` (both optional): routing weights [T*k] bf16 and their
// fp32 copies in sorted-row order, for the fused down-projection combine.
int launch_permute(const int32_t* idx, int64_t T, int k, int64_t E, int64_t capacity,
                   int32_t* sorted_token, int32_t* inv_pos, int32_t* group_sizes,
                   int32_t* group_offsets, cudaStream_t stream, const void* w = nullptr,
                   float* sorted_w = nullptr);
// Multi-block version of launch_permute (same outputs) for callers with
// scratch: `hist` holds permute_hist_ints(E) ints.  With `active` (E + 1
// ints, optional) it also lists the experts that kept rows: active[0] =
// their count, active[1..] = the experts in increasing order.
constexpr int kPermMaxBlocks = 148;
int64_t permute_hist_ints(int64_t E);
int launch_permute_multi(const int32_t* idx, int64_t T, int k, int64_t E, int64_t capacity,
                         int32_t* hist, int32_t* sorted_token, int32_t* inv_pos,
                         int32_t* group_sizes, int32_t* group_offsets, cudaStream_t stream,
                         const void* w, float* sorted_w, int32_t* active = nullptr);
int launch_f32_to_bf16(const float* acc, int64_t n, void* out, cudaStream_t stream);
int launch_build_tiles(const int32_t* group_offsets, int64_t E, int nt, TileEntry* tiles,
                       int32_t* num_tiles, cudaStream_t stream);
int launch_gather(const void* x, const int32_t* sorted_token, const int32_t* total_rows,
                  int64_t max_rows, int64_t D, void* xs, cudaStream_t stream);
// out [T][D]: bf16, or fp32 with out_f32 (the k rows summed in slot order).
int launch_combine(const void* ys, const int32_t* inv_pos, const void* w, int64_t T, int k,
                   int64_t D, void* out, cudaStream_t stream, bool out_f32 = false);

}  // namespace kw8
