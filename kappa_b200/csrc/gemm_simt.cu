// Grouped W8A16 GEMV for few tokens per group (decode).
//
// Streams each weight row once from HBM with 16-byte non-allocating loads,
// widens int8 to fp32 in registers and multiplies it with up to kTN token
// rows of the group (fp32 accumulate).  One warp per output feature (paired
// mode: the gate row and the up row of that feature); 8 warps per CTA.
// Grid: x = feature blocks of 8, y = tile-table entries (an upper bound;
// surplus CTAs exit).  Used when a group holds at most a few tokens, where
// the work is bound by weight bytes, not by arithmetic.
#include "gemm_simt.cuh"

namespace kw8 {

namespace {

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// 16 int8 -> 16 fp32, exact: each byte q is biased to u = q + 128, placed
// in the mantissa of the fp32 2^23 (bits 0x4B0000uu = 8388608 + u), and
// 8388608 + 128 is subtracted.
__device__ __forceinline__ void i8x16_to_f32(const uint4& w, float* f) {
  const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t u = words[i] ^ 0x80808080u;
    f[4 * i + 0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - 8388736.0f;
    f[4 * i + 1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - 8388736.0f;
    f[4 * i + 2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - 8388736.0f;
    f[4 * i + 3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - 8388736.0f;
  }
}

__device__ __forceinline__ void bf16x8_to_f32(const uint4& v, float* f) {
  const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i + 0] = __uint_as_float(words[i] << 16);
    f[2 * i + 1] = __uint_as_float(words[i] & 0xFFFF0000u);
  }
}

template <int kMode, int kTN>
__global__ void __launch_bounds__(256)
    w8_gemm_simt_kernel(const int8_t* __restrict__ wa, const int8_t* __restrict__ wb,
                        const __nv_bfloat16* __restrict__ x, int64_t ldx, GemmArgs p) {
  constexpr bool kPair = epi_is_pair(kMode);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int entry = blockIdx.y;
  int group, row0, nrows;
  if (p.tiles == nullptr) {
    group = 0;
    row0 = entry * kTN;
    if (row0 >= p.dense_rows) return;
    nrows = min(kTN, p.dense_rows - row0);
  } else {
    if (entry >= *p.num_tiles) return;
    const TileEntry te = p.tiles[entry];
    group = te.group;
    row0 = te.row0;
    nrows = te.nrows;
  }
  const int f = blockIdx.x * 8 + warp;
  if (f >= p.N_out) return;
  const int64_t wrow = (static_cast<int64_t>(group) * p.N_out + f) * p.K;
  const int8_t* ra = wa + wrow;
  const int8_t* rb = kPair ? wb + wrow : nullptr;

  float acc_a[kTN], acc_b[kTN];
#pragma unroll
  for (int t = 0; t < kTN; ++t) acc_a[t] = acc_b[t] = 0.f;

  for (int k0 = lane * 16; k0 < p.K; k0 += 32 * 16) {
    float wfa[16], wfb[16];
    i8x16_to_f32(ld_nc_v4(ra + k0), wfa);
    if (kPair) i8x16_to_f32(ld_nc_v4(rb + k0), wfb);
#pragma unroll
    for (int t = 0; t < kTN; ++t) {
      if (t < nrows) {
        const __nv_bfloat16* xr = x + static_cast<int64_t>(row0 + t) * ldx + k0;
        float xf[16];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(xr), xf);
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(xr + 8), xf + 8);
        float sa = 0.f, sb = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          sa = fmaf(wfa[i], xf[i], sa);
          if (kPair) sb = fmaf(wfb[i], xf[i], sb);
        }
        acc_a[t] += sa;
        if (kPair) acc_b[t] += sb;
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kTN; ++t) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc_a[t] += __shfl_xor_sync(0xffffffffu, acc_a[t], o);
      if (kPair) acc_b[t] += __shfl_xor_sync(0xffffffffu, acc_b[t], o);
    }
  }
  const int64_t sidx = static_cast<int64_t>(group) * p.N_out + f;
  const float s_a = load_scale(p.scale_a, p.scale_a_dtype, p.scale_a_pc ? sidx : 0);
  float s_b = 0.f;
  if (kPair) s_b = load_scale(p.scale_b, p.scale_b_dtype, p.scale_b_pc ? sidx : 0);
  // Lane t writes token t.
#pragma unroll
  for (int t = 0; t < kTN; ++t) {
    if (lane == t && t < nrows) {
      const int64_t o = static_cast<int64_t>(row0 + t) * p.ld_out + f;
      if constexpr (kPair) {
        const float g = acc_a[t] * s_a, u = acc_b[t] * s_b;
        const float h = (kMode == EPI_PAIR_GELU) ? gelu_tanh_f(g) * u : silu_f(g) * u;
        static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(h);
      } else if constexpr (kMode == EPI_COMBINE_F32) {
        const int r = row0 + t;
        atomicAdd(static_cast<float*>(p.out) + static_cast<int64_t>(p.row_token[r]) * p.ld_out + f,
                  acc_a[t] * s_a * p.row_weight[r]);
      } else if constexpr (kMode == EPI_PLAIN_F32) {
        static_cast<float*>(p.out)[o] = acc_a[t] * s_a;
      } else {
        static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(acc_a[t] * s_a);
      }
    }
  }
}

template <int kMode>
int launch_simt_mode(const int8_t* wa, const int8_t* wb, const void* x, int64_t ldx,
                     const GemmArgs& args, int64_t max_entries, cudaStream_t stream) {
  dim3 grid(static_cast<unsigned>((args.N_out + 7) / 8), static_cast<unsigned>(max_entries));
  w8_gemm_simt_kernel<kMode, kSimtTN><<<grid, 256, 0, stream>>>(
      wa, wb, static_cast<const __nv_bfloat16*>(x), ldx, args);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

}  // namespace

int launch_gemm_simt(int mode, const int8_t* wa, const int8_t* wb, int64_t groups,
                     int64_t N_out, int64_t K, const void* x, int64_t x_rows, int64_t ldx,
                     const GemmArgs& args_in, cudaStream_t stream) {
  const bool pair = epi_is_pair(mode);
  KW8_REQUIRE(K > 0 && K % 16 == 0, KW8_ERR_UNSUPPORTED, "K=%lld must be a positive multiple of 16",
              (long long)K);
  KW8_REQUIRE(ldx % 8 == 0 && ldx >= K, KW8_ERR_UNSUPPORTED, "token row pitch invalid");
  KW8_REQUIRE(!pair || wb != nullptr, KW8_ERR_INVALID_ARG, "paired GEMV needs two weights");
  KW8_REQUIRE(args_in.nt == kSimtTN, KW8_ERR_INVALID_ARG, "GEMV token tile must be %d", kSimtTN);
  KW8_REQUIRE(groups * N_out < (1ll << 31), KW8_ERR_UNSUPPORTED, "weight rows out of range");
  GemmArgs args = args_in;
  args.K = static_cast<int>(K);
  args.N_out = static_cast<int>(N_out);
  args.m_tiles = 1;
  const int64_t max_entries = args.tiles == nullptr ? (args.dense_rows + kSimtTN - 1) / kSimtTN
                                                    : groups + (x_rows + kSimtTN - 1) / kSimtTN;
  if (max_entries <= 0) return KW8_OK;
  KW8_REQUIRE(max_entries < 65536, KW8_ERR_UNSUPPORTED, "too many GEMV tiles");
  switch (mode) {
    case EPI_PAIR_GELU:
      return launch_simt_mode<EPI_PAIR_GELU>(wa, wb, x, ldx, args, max_entries, stream);
    case EPI_PAIR_SILU:
      return launch_simt_mode<EPI_PAIR_SILU>(wa, wb, x, ldx, args, max_entries, stream);
    case EPI_PLAIN_BF16:
      return launch_simt_mode<EPI_PLAIN_BF16>(wa, wb, x, ldx, args, max_entries, stream);
    case EPI_PLAIN_F32:
      return launch_simt_mode<EPI_PLAIN_F32>(wa, wb, x, ldx, args, max_entries, stream);
    case EPI_COMBINE_F32:
      KW8_REQUIRE(args.row_token && args.row_weight, KW8_ERR_INVALID_ARG, "combine needs row maps");
      return launch_simt_mode<EPI_COMBINE_F32>(wa, wb, x, ldx, args, max_entries, stream);
    default:
      return fail(KW8_ERR_INVALID_ARG, "unknown epilogue mode %d", mode);
  }
}

}  // namespace kw8
