// RMSNorm and the residual epilogue of a decoder block's FFN (see norm.cu).
#pragma once

#include "common.cuh"

namespace kw8 {

// Rows of D (a multiple of 8, at most kNormMaxD) spread over CTAs of
// kNormThreads threads, each thread holding at most kNormMaxVec 8-wide vectors.
constexpr int kNormThreads = 256;
constexpr int kNormMaxVec = 8;  // 8-wide vectors per thread
constexpr int64_t kNormMaxD = static_cast<int64_t>(kNormThreads) * 8 * kNormMaxVec;

// out = bf16((f32(x) * rsqrt(mean(f32(x)^2) + eps)) * g), g = 1 + scale
// (kind KW8_NORM_GEMMA) or scale (KW8_NORM_QWEN); x, out bf16 [T][D].
int launch_rms_norm(const void* x, int64_t T, int64_t D, const void* scale, int scale_dtype,
                    int kind, float eps, void* out, cudaStream_t stream);

// The end of the FFN sub-block, row by row:
//   y   = bf16(sum over s < splits of part[s][t])   (the FFN output, fp32 partials)
//   y   = rms_norm(y, post_scale)                   (if post_scale != nullptr)
//   out = bf16(f32(h[t]) + f32(y))                  (if h != nullptr; else out = y)
int launch_block_finish(const float* part, int splits, int64_t split_stride, int64_t T, int64_t D,
                        const void* post_scale, int scale_dtype, int kind, float eps,
                        const void* h, void* out, cudaStream_t stream);

}  // namespace kw8
