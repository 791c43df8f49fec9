// RMSNorm (kappa/gemma3/norms.py:8-13 with Gemma's (1 + scale),
// kappa/qwen3/norms.py:10-16 with Qwen's scale) and the residual epilogue of
// the FFN sub-block (kappa/gemma3/block.py:73-82, kappa/qwen3/block.py:68-81).
//
// A CTA takes up to 256 / tpr rows, tpr threads per row (the fewest, from
// 32, that hold the row in at most kNormMaxVec 8-wide vectors each: one
// warp per 2048-wide row), fewer rows when the grid would otherwise have
// under two CTAs per SM.  The row is read once into registers,
// the sum of squares is reduced over the row's threads in fp32 (a fixed
// order), and the row is written once.  Rounding follows kappa: the norm computes in fp32 and rounds its
// output to the activation dtype once; the FFN output is rounded to bf16
// before the post-FFN norm, and the residual add rounds once more.
#include "norm.cuh"

namespace kw8 {

namespace {

// Sum of v over the tpr threads of this thread's row group (every thread
// of the CTA calls it; the result is the same in every thread of a group).
__device__ __forceinline__ float group_sum(float v, float* red, int tpr) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if (tpr == 32) return v;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read by an earlier call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int wpg = tpr >> 5, first = (warp / wpg) * wpg;
  float s = 0.f;
  for (int w = 0; w < wpg; ++w) s += red[first + w];  // the same order in every thread
  return s;
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint4 f32x8_to_bf16(const float (&f)[8]) {
  uint4 o;
  uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    ow[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  return o;
}

// g[d] of the norm: 1 + scale (Gemma) or scale (Qwen), in fp32.
__device__ __forceinline__ float norm_gain(const void* scale, int dtype, int kind, int64_t d) {
  const float s = load_scale(scale, dtype, d);
  return kind == KW8_NORM_GEMMA ? 1.0f + s : s;
}

// v (this thread's nv vectors of the row, fp32) <- (v * r) * g, r from the
// row's mean square.
__device__ __forceinline__ void rms_apply(float (&v)[kNormMaxVec][8], int nv, int64_t D,
                                          const void* scale, int dtype, int kind, float eps,
                                          float* red, int tpr, int tl) {
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j)
    if (j < nv)
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(v[j][i], v[j][i], ss);
  const float total = group_sum(ss, red, tpr);
  const float r = rsqrtf(__fdiv_rn(total, static_cast<float>(D)) + eps);
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    if (j >= nv) continue;
    const int64_t d0 = (static_cast<int64_t>(j) * tpr + tl) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) v[j][i] = __fmul_rn(__fmul_rn(v[j][i], r), norm_gain(scale, dtype, kind, d0 + i));
  }
}

__global__ void __launch_bounds__(kNormThreads)
    rms_norm_kernel(const uint4* __restrict__ x, int64_t T, int64_t D, const void* __restrict__ scale, int dtype,
                    int kind, float eps, int tpr, uint4* __restrict__ out) {
  __shared__ float red[kNormThreads / 32];
  const int64_t vec = D / 8;
  const int tl = threadIdx.x % tpr;
  const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x / tpr) + threadIdx.x / tpr;
  const int nv = row < T ? static_cast<int>((vec - tl + tpr - 1) / tpr) : 0;
  const uint4* xr = x + row * vec;
  float v[kNormMaxVec][8];
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j)
    if (j < nv) bf16x8_to_f32(xr[j * tpr + tl], v[j]);
  rms_apply(v, nv, D, scale, dtype, kind, eps, red, tpr, tl);
  uint4* orow = out + row * vec;
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j)
    if (j < nv) orow[j * tpr + tl] = f32x8_to_bf16(v[j]);
}

__global__ void __launch_bounds__(kNormThreads)
    block_finish_kernel(const float4* __restrict__ part, int splits, int64_t stride4, int64_t T, int64_t D,
                        const void* __restrict__ scale, int dtype, int kind, float eps,
                        const uint4* __restrict__ h, int tpr, uint4* __restrict__ out) {
  __shared__ float red[kNormThreads / 32];
  const int64_t vec = D / 8;
  const int tl = threadIdx.x % tpr;
  const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x / tpr) + threadIdx.x / tpr;
  const int nv = row < T ? static_cast<int>((vec - tl + tpr - 1) / tpr) : 0;
  float v[kNormMaxVec][8];
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    if (j >= nv) continue;
    const int64_t e4 = (row * vec + j * tpr + tl) * 2;  // float4 index
    float4 a = part[e4], b = part[e4 + 1];
    for (int s = 1; s < splits; ++s) {
      const float4 c = part[s * stride4 + e4], d = part[s * stride4 + e4 + 1];
      a.x += c.x; a.y += c.y; a.z += c.z; a.w += c.w;
      b.x += d.x; b.y += d.y; b.z += d.z; b.w += d.w;
    }
    const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) v[j][i] = __bfloat162float(__float2bfloat16_rn(f[i]));  // the FFN output in bf16
  }
  if (scale != nullptr) {
    rms_apply(v, nv, D, scale, dtype, kind, eps, red, tpr, tl);
#pragma unroll
    for (int j = 0; j < kNormMaxVec; ++j)
      if (j < nv)
#pragma unroll
        for (int i = 0; i < 8; ++i) v[j][i] = __bfloat162float(__float2bfloat16_rn(v[j][i]));
  }
#pragma unroll
  for (int j = 0; j < kNormMaxVec; ++j) {
    if (j >= nv) continue;
    const int64_t e = row * vec + j * tpr + tl;
    if (h != nullptr) {
      float hv[8];
      bf16x8_to_f32(h[e], hv);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[j][i] = __fadd_rn(hv[i], v[j][i]);
    }
    out[e] = f32x8_to_bf16(v[j]);
  }
}

// Threads per row: the fewest of 32, 64, 128, 256 that hold a row in at most
// kNormMaxVec vectors each, doubled while the rows would keep fewer than
// ~131k threads busy (few rows: more threads per row; measured at T = 256 /
// 4096, D = 2560 / 2048).
int norm_tpr(int64_t T, int64_t D) {
  const int64_t vec = D / 8;
  int tpr = 32;
  while (tpr < kNormThreads && (vec + tpr - 1) / tpr > kNormMaxVec) tpr *= 2;
  while (tpr < kNormThreads && tpr < vec && T * tpr < 148 * 896) tpr *= 2;
  return tpr;
}

// Rows per CTA: as many as kNormThreads threads hold, fewer when that would
// leave fewer than two CTAs per SM (few rows: T = 256 gets one row a CTA).
int64_t norm_rows_per_cta(int64_t T, int tpr) {
  int64_t rpc = kNormThreads / tpr;
  while (rpc > 1 && (T + rpc - 1) / rpc < 2 * 148) rpc /= 2;
  return rpc;
}

int check_norm(int64_t T, int64_t D, int scale_dtype, int kind, float eps) {
  KW8_REQUIRE(T >= 0 && D >= 8 && D % 8 == 0 && D <= kNormMaxD, KW8_ERR_UNSUPPORTED,
              "RMSNorm rows need D %% 8 == 0 and 8 <= D <= %lld (D=%lld)", (long long)kNormMaxD,
              (long long)D);
  KW8_REQUIRE(T < (1ll << 31), KW8_ERR_UNSUPPORTED, "too many rows");
  KW8_REQUIRE(scale_dtype == KW8_DT_F32 || scale_dtype == KW8_DT_BF16, KW8_ERR_INVALID_ARG,
              "norm scale dtype must be f32 or bf16");
  KW8_REQUIRE(kind == KW8_NORM_GEMMA || kind == KW8_NORM_QWEN, KW8_ERR_INVALID_ARG, "unknown norm kind %d",
              kind);
  KW8_REQUIRE(eps >= 0.f, KW8_ERR_INVALID_ARG, "eps must be >= 0");
  return KW8_OK;
}

}  // namespace

int launch_rms_norm(const void* x, int64_t T, int64_t D, const void* scale, int scale_dtype, int kind,
                    float eps, void* out, cudaStream_t stream) {
  KW8_REQUIRE(x && scale && out, KW8_ERR_INVALID_ARG, "null pointer");
  int rc = check_norm(T, D, scale_dtype, kind, eps);
  if (rc) return rc;
  KW8_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) & 15) == 0,
              KW8_ERR_UNSUPPORTED, "RMSNorm rows must be 16-byte aligned");
  if (T == 0) return KW8_OK;
  const int tpr = norm_tpr(T, D);
  const int64_t rpc = norm_rows_per_cta(T, tpr);
  rms_norm_kernel<<<static_cast<unsigned>((T + rpc - 1) / rpc), static_cast<unsigned>(rpc * tpr), 0, stream>>>(
      static_cast<const uint4*>(x), T, D, scale, scale_dtype, kind, eps, tpr, static_cast<uint4*>(out));
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_block_finish(const float* part, int splits, int64_t split_stride, int64_t T, int64_t D,
                        const void* post_scale, int scale_dtype, int kind, float eps, const void* h,
                        void* out, cudaStream_t stream) {
  KW8_REQUIRE(part && out && splits >= 1, KW8_ERR_INVALID_ARG, "null pointer");
  int rc = check_norm(T, D, scale_dtype, kind, eps);
  if (rc) return rc;
  KW8_REQUIRE(split_stride % 4 == 0 &&
                  ((reinterpret_cast<uintptr_t>(part) | reinterpret_cast<uintptr_t>(out) |
                    reinterpret_cast<uintptr_t>(h)) & 15) == 0,
              KW8_ERR_UNSUPPORTED, "block epilogue rows must be 16-byte aligned");
  if (T == 0) return KW8_OK;
  const int tpr = norm_tpr(T, D);
  const int64_t rpc = norm_rows_per_cta(T, tpr);
  block_finish_kernel<<<static_cast<unsigned>((T + rpc - 1) / rpc), static_cast<unsigned>(rpc * tpr), 0, stream>>>(
      reinterpret_cast<const float4*>(part), splits, split_stride / 4, T, D, post_scale, scale_dtype, kind, eps,
      static_cast<const uint4*>(h), tpr, static_cast<uint4*>(out));
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

}  // namespace kw8
