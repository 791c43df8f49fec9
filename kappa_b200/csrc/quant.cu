// W8 quantisation (kappa/qwen3/quant.py:41-48) and dequantisation
// (quant.py:34-38) kernels.
//
// quantize: pass 1 takes the absmax of every output channel (a warp per
// channel when K is contiguous; a thread per channel and 64-k chunk when
// the channels are contiguous) and, for the per-tensor form, folds it into
// one word
// with an integer atomicMax on the float's bits (valid for non-negative
// floats; max is order independent, so the result is deterministic).
// Pass 2 computes scale = max(amax / 127, FLT_MIN) with IEEE division,
// q = clip(rint(w / scale), -128, 127) (rintf rounds half to even, like
// jnp.round) and writes q K-major; the stored scale is the fp32 scale
// rounded to nearest even in the requested dtype.
#include "quant.cuh"

namespace kw8 {

namespace {

__device__ __forceinline__ float load_w(const void* w, int dtype, int64_t i) {
  if (dtype == KW8_DT_F32) return static_cast<const float*>(w)[i];
  return bf16_bits_to_f32(static_cast<const uint16_t*>(w)[i]);
}

// A thread per output channel walking K: coalesced across threads when the
// channels are contiguous (sn == 1, N-contiguous input).
__global__ void amax_kernel(const void* __restrict__ w, int dtype, int64_t outer, int64_t K,
                            int64_t N, int64_t so, int64_t sk, int64_t sn, int per_channel,
                            float* __restrict__ ch_amax, unsigned* __restrict__ glob) {
  const int64_t ch = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (ch >= outer * N) return;
  const int64_t o = ch / N, n = ch - o * N;
  const int64_t base = o * so + n * sn;
  float m = 0.f;
  for (int64_t k = 0; k < K; ++k) m = fmaxf(m, fabsf(load_w(w, dtype, base + k * sk)));
  if (per_channel)
    ch_amax[ch] = m;
  else
    atomicMax(glob, __float_as_uint(m));
}

// Channels contiguous (sn == 1): a thread per channel and 64-k chunk, the
// threads of a warp reading 32 consecutive channels; chunk maxima combine
// with an integer atomicMax on the float's bits (values are >= 0, so the
// order of the bits is the order of the values; ch_amax starts at zero).
constexpr int64_t kAmaxChunk = 64;
__global__ void amax_cols_kernel(const void* __restrict__ w, int dtype, int64_t outer, int64_t K,
                                 int64_t N, int64_t so, int64_t sk, int per_channel,
                                 unsigned* __restrict__ ch_amax_bits, unsigned* __restrict__ glob) {
  const int64_t ch = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (ch >= outer * N) return;
  const int64_t o = ch / N, n = ch - o * N;
  const int64_t base = o * so + n;
  const int64_t k0 = static_cast<int64_t>(blockIdx.y) * kAmaxChunk;
  const int64_t k1 = k0 + kAmaxChunk < K ? k0 + kAmaxChunk : K;
  float m = 0.f;
  for (int64_t k = k0; k < k1; ++k) m = fmaxf(m, fabsf(load_w(w, dtype, base + k * sk)));
  atomicMax(per_channel ? ch_amax_bits + ch : glob, __float_as_uint(m));
}

// A warp per output channel with K contiguous (sk == 1): the lanes read
// consecutive k and reduce with shuffles (max is order independent, so the
// result equals the serial walk's).
__global__ void amax_rows_kernel(const void* __restrict__ w, int dtype, int64_t outer, int64_t K,
                                 int64_t N, int64_t so, int64_t sn, int per_channel,
                                 float* __restrict__ ch_amax, unsigned* __restrict__ glob) {
  const int lane = threadIdx.x & 31;
  const int64_t ch = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  if (ch >= outer * N) return;  // uniform over the warp
  const int64_t o = ch / N, n = ch - o * N;
  const int64_t base = o * so + n * sn;
  float m = 0.f;
  for (int64_t k = lane; k < K; k += 32) m = fmaxf(m, fabsf(load_w(w, dtype, base + k)));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane != 0) return;
  if (per_channel)
    ch_amax[ch] = m;
  else
    atomicMax(glob, __float_as_uint(m));
}

__device__ __forceinline__ float scale_from_amax(float amax) {
  return fmaxf(__fdiv_rn(amax, 127.0f), 1.17549435e-38f);  // FLT_MIN floor
}

__device__ __forceinline__ int8_t quant1(float w, float s) {
  float r = rintf(__fdiv_rn(w, s));
  r = fminf(fmaxf(r, -128.0f), 127.0f);
  return static_cast<int8_t>(static_cast<int>(r));
}

// One thread per (outer, n, 16-wide k chunk); writes 16 bytes of q[o][n][k].
// `k_fast` selects the thread order: consecutive threads take consecutive k
// chunks (K-contiguous input) or consecutive channels (N-contiguous input).
__global__ void quant_kernel(const void* __restrict__ w, int dtype, int64_t outer, int64_t K,
                             int64_t N, int64_t so, int64_t sk, int64_t sn, int per_channel,
                             const float* __restrict__ ch_amax, const unsigned* __restrict__ glob,
                             int k_fast, int scale_dtype, int8_t* __restrict__ q,
                             void* __restrict__ scale_out) {
  const int64_t kc = (K + 15) / 16;
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (tid >= outer * N * kc) return;
  int64_t ch, c;
  if (k_fast) {
    ch = tid / kc;
    c = tid - ch * kc;
  } else {
    const int64_t on = outer * N;
    c = tid / on;
    ch = tid - c * on;
  }
  const int64_t o = ch / N, n = ch - o * N;
  const float amax = per_channel ? ch_amax[ch] : __uint_as_float(*glob);
  const float s = scale_from_amax(amax);
  const int64_t base = o * so + n * sn;
  alignas(16) int8_t buf[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int64_t k = c * 16 + i;
    buf[i] = (k < K) ? quant1(load_w(w, dtype, base + k * sk), s) : 0;
  }
  int8_t* dst = q + ch * K + c * 16;
  if (K % 16 == 0) {
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(buf);
  } else {
    for (int i = 0; i < 16 && c * 16 + i < K; ++i) dst[i] = buf[i];
  }
  const bool writer = per_channel ? (c == 0) : (tid == 0);
  if (writer) {
    const int64_t si = per_channel ? ch : 0;
    if (scale_dtype == KW8_DT_F32)
      static_cast<float*>(scale_out)[si] = s;
    else
      static_cast<__nv_bfloat16*>(scale_out)[si] = __float2bfloat16_rn(s);
  }
}

__global__ void dequant_kernel(const int8_t* __restrict__ q, const void* __restrict__ scale,
                               int scale_dtype, int per_channel, int64_t K, int64_t total,
                               int out_dtype, void* __restrict__ out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float s = load_scale(scale, scale_dtype, per_channel ? i / K : 0);
    const float v = static_cast<float>(q[i]);
    if (out_dtype == KW8_DT_F32) {
      static_cast<float*>(out)[i] = v * s;  // exact: 8-bit x 8..24-bit mantissa
    } else {
      // bf16(q) * bf16(s) rounded once to bf16; q and bf16(s) are exact in
      // fp32 and so is their product (<= 16 significant bits).
      const float sb = __bfloat162float(__float2bfloat16_rn(s));
      static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v * sb);
    }
  }
}

// gather_embed_tokens: out[i][d] = dt(q[row][d]) * dt(s) for row = tokens[i]
// normalised like a JAX gather (negative ids count from the end, then the
// id is clamped into [0, V)).  One rounding per product, as dequant_kernel.
// A thread per 8 outputs (8 int8 in, 8 bf16 / fp32 out).
__global__ void embed_gather_kernel(const int32_t* __restrict__ tokens, int64_t n,
                                    const int8_t* __restrict__ q, const void* __restrict__ scale,
                                    int scale_dtype, int per_channel, int64_t V, int64_t D,
                                    int out_dtype, void* __restrict__ out) {
  const int64_t vec = D / 8;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n * vec;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / vec, c = i - t * vec;
    int64_t row = tokens[t];
    if (row < 0) row += V;
    row = row < 0 ? 0 : (row >= V ? V - 1 : row);
    float s = load_scale(scale, scale_dtype, per_channel ? row : 0);
    if (out_dtype == KW8_DT_BF16) s = __bfloat162float(__float2bfloat16_rn(s));
    const uint2 w = *reinterpret_cast<const uint2*>(q + row * D + c * 8);
    const uint32_t words[2] = {w.x, w.y};
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = static_cast<float>(static_cast<int8_t>((words[j >> 2] >> (8 * (j & 3))) & 0xFFu)) * s;
    if (out_dtype == KW8_DT_F32) {
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + t * D + c * 8);
      o[0] = make_float4(v[0], v[1], v[2], v[3]);
      o[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
        ow[j] = *reinterpret_cast<const uint32_t*>(&b);
      }
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + t * D + c * 8) = o;
    }
  }
}

}  // namespace

int launch_embed_gather(const int32_t* tokens, int64_t n, const kw8_weight& table, int64_t V,
                        int64_t D, int out_dtype, void* out, cudaStream_t stream) {
  KW8_REQUIRE(tokens && table.q && table.scale && out, KW8_ERR_INVALID_ARG, "null pointer");
  KW8_REQUIRE(n >= 0 && V >= 1 && D >= 1, KW8_ERR_INVALID_ARG, "bad shape (n=%lld V=%lld D=%lld)",
              (long long)n, (long long)V, (long long)D);
  KW8_REQUIRE(out_dtype == KW8_DT_F32 || out_dtype == KW8_DT_BF16, KW8_ERR_INVALID_ARG,
              "out dtype must be f32 or bf16");
  KW8_REQUIRE(D % 8 == 0 && (reinterpret_cast<uintptr_t>(table.q) & 7) == 0 &&
                  (reinterpret_cast<uintptr_t>(out) & 15) == 0,
              KW8_ERR_UNSUPPORTED, "embedding rows need D %% 8 == 0 and aligned buffers");
  if (n == 0) return KW8_OK;
  int64_t blocks = (n * (D / 8) + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  embed_gather_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      tokens, n, table.q, table.scale, table.scale_dtype, table.per_channel, V, D, out_dtype, out);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

size_t quantize_workspace_size(int64_t outer, int64_t N) {
  return static_cast<size_t>(outer * N + 4) * sizeof(float);
}

int launch_quantize(const void* w, int w_dtype, int64_t outer, int64_t K, int64_t N, int64_t so,
                    int64_t sk, int64_t sn, int per_channel, int scale_dtype, int8_t* q,
                    void* scale_out, void* ws, size_t ws_bytes, cudaStream_t stream) {
  KW8_REQUIRE(w && q && scale_out, KW8_ERR_INVALID_ARG, "null pointer");
  KW8_REQUIRE(outer >= 1 && K >= 1 && N >= 1, KW8_ERR_INVALID_ARG, "empty weight");
  KW8_REQUIRE(w_dtype == KW8_DT_F32 || w_dtype == KW8_DT_BF16, KW8_ERR_INVALID_ARG,
              "weight dtype must be f32 or bf16");
  KW8_REQUIRE(scale_dtype == KW8_DT_F32 || scale_dtype == KW8_DT_BF16, KW8_ERR_INVALID_ARG,
              "scale dtype must be f32 or bf16");
  KW8_REQUIRE(ws != nullptr && ws_bytes >= quantize_workspace_size(outer, N), KW8_ERR_WORKSPACE,
              "quantize workspace too small (%zu < %zu)", ws_bytes,
              quantize_workspace_size(outer, N));
  KW8_REQUIRE((reinterpret_cast<uintptr_t>(q) & 15) == 0 || K % 16 != 0, KW8_ERR_INVALID_ARG,
              "q_out must be 16-byte aligned");
  float* ch_amax = static_cast<float*>(ws);
  unsigned* glob = reinterpret_cast<unsigned*>(ch_amax + outer * N);
  KW8_CUDA_TRY(cudaMemsetAsync(glob, 0, sizeof(unsigned), stream));
  const int64_t channels = outer * N;
  if (sk == 1) {  // K contiguous: a warp per channel
    amax_rows_kernel<<<static_cast<unsigned>((channels * 32 + 255) / 256), 256, 0, stream>>>(
        w, w_dtype, outer, K, N, so, sn, per_channel, ch_amax, glob);
  } else if (sn == 1 && (K + kAmaxChunk - 1) / kAmaxChunk <= 65535) {  // channels contiguous: split K too
    if (per_channel) KW8_CUDA_TRY(cudaMemsetAsync(ch_amax, 0, static_cast<size_t>(channels) * sizeof(float), stream));
    const dim3 grid(static_cast<unsigned>((channels + 255) / 256),
                    static_cast<unsigned>((K + kAmaxChunk - 1) / kAmaxChunk));
    amax_cols_kernel<<<grid, 256, 0, stream>>>(w, w_dtype, outer, K, N, so, sk, per_channel,
                                               reinterpret_cast<unsigned*>(ch_amax), glob);
  } else {
    amax_kernel<<<static_cast<unsigned>((channels + 255) / 256), 256, 0, stream>>>(
        w, w_dtype, outer, K, N, so, sk, sn, per_channel, ch_amax, glob);
  }
  KW8_CHECK_LAUNCH();
  const int64_t threads = channels * ((K + 15) / 16);
  const int k_fast = (sk == 1) ? 1 : 0;
  quant_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(
      w, w_dtype, outer, K, N, so, sk, sn, per_channel, ch_amax, glob, k_fast, scale_dtype, q,
      scale_out);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_dequantize(const kw8_weight& w, int64_t groups, int64_t N, int64_t K, int out_dtype,
                      void* out, cudaStream_t stream) {
  KW8_REQUIRE(w.q && w.scale && out, KW8_ERR_INVALID_ARG, "null pointer");
  KW8_REQUIRE(out_dtype == KW8_DT_F32 || out_dtype == KW8_DT_BF16, KW8_ERR_INVALID_ARG,
              "out dtype must be f32 or bf16");
  const int64_t total = groups * N * K;
  if (total <= 0) return KW8_OK;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  dequant_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      w.q, w.scale, w.scale_dtype, w.per_channel, K, total, out_dtype, out);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

}  // namespace kw8
