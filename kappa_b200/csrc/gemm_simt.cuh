// Grouped W8A16 GEMV for few tokens per group (see gemm_simt.cu).
#pragma once

#include "gemm_tc.cuh"

namespace kw8 {

constexpr int kSimtTN = 8;  // token rows per GEMV tile

int launch_gemm_simt(int mode, const int8_t* wa, const int8_t* wb, int64_t groups,
                     int64_t N_out, int64_t K, const void* x, int64_t x_rows, int64_t ldx,
                     const GemmArgs& args_in, cudaStream_t stream);

}  // namespace kw8
