// Pre-packed ("tiled") W8 weight layout, produced once at load time.
//
// A K-major weight [groups][N][K] int8 is stored as
//   [groups][FT = ceil(N / 16)][KS = ceil(K / 128) * 2][1024 bytes]
// (K padded with zeros to a multiple of 128, N to a multiple of 16).  Block
// (g, f, s) holds rows 16f .. 16f + 15 and k = 64s .. 64s + 63; row
// 16f + 8h + r (h = 0, 1; r = 0..7) and the 16 k of chunk c (c = 0..3) sit
// at byte 512 h + 16 (8 c + r).  So
//   * the weight-streaming kernel's warp (lane (r, c) holds row r and row
//     r + 8, chunk c of a 64-k step) reads each step as two 512-byte
//     contiguous pieces, one 16-byte copy per lane each (a row-major weight
//     gives 32 pieces of 64 bytes in 32 rows);
//   * the tensor-core kernel's stage (128 rows x 128 k) is 8 feature tiles
//   x 2 steps: one 3-D TMA box (256 B x 8 x 8), and its converters (a
//     thread per row) read 8 consecutive rows' chunks as 128 contiguous
//     bytes (no shared-memory bank conflicts).
#include "pack.cuh"

namespace kw8 {

namespace {

// One thread per (group, feature tile, step, chunk position 0..63): the 16
// bytes of row 16f + 8h + r, k = 64s + 16c .. +15 (zero past N or K).
__global__ void pack_kernel(const int8_t* __restrict__ q, int64_t groups, int64_t N, int64_t K, int64_t FT,
                            int64_t KS, uint4* __restrict__ out) {
  const int64_t total = groups * FT * KS * 64;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int pos = static_cast<int>(i & 63);  // 16-byte unit within the 1 KB block
    int64_t blk = i >> 6;
    const int64_t s = blk % KS;
    blk /= KS;
    const int64_t f = blk % FT;
    const int64_t g = blk / FT;
    const int h = pos >> 5, c = (pos >> 3) & 3, r = pos & 7;
    const int64_t n = 16 * f + 8 * h + r;
    const int64_t k0 = 64 * s + 16 * c;
    alignas(16) int8_t b[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      b[j] = (n < N && k0 + j < K) ? q[(g * N + n) * K + k0 + j] : static_cast<int8_t>(0);
    out[i] = *reinterpret_cast<const uint4*>(b);
  }
}

// The inverse: tiled -> K-major [groups][N][K].
__global__ void unpack_kernel(const uint4* __restrict__ t, int64_t groups, int64_t N, int64_t K, int64_t FT,
                              int64_t KS, int8_t* __restrict__ q) {
  const int64_t total = groups * FT * KS * 64;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int pos = static_cast<int>(i & 63);
    int64_t blk = i >> 6;
    const int64_t s = blk % KS;
    blk /= KS;
    const int64_t f = blk % FT;
    const int64_t g = blk / FT;
    const int h = pos >> 5, c = (pos >> 3) & 3, r = pos & 7;
    const int64_t n = 16 * f + 8 * h + r;
    const int64_t k0 = 64 * s + 16 * c;
    if (n >= N) continue;
    alignas(16) int8_t b[16];
    *reinterpret_cast<uint4*>(b) = t[i];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (k0 + j < K) q[(g * N + n) * K + k0 + j] = b[j];
  }
}

int pack_grid(int64_t n) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 148 * 16)));
}

}  // namespace

int launch_pack(const int8_t* q, int64_t groups, int64_t N, int64_t K, void* out, cudaStream_t stream) {
  KW8_REQUIRE(q && out, KW8_ERR_INVALID_ARG, "null pointer");
  KW8_REQUIRE(groups >= 1 && N >= 1 && K >= 1 && K % 16 == 0, KW8_ERR_INVALID_ARG,
              "bad weight shape (groups=%lld N=%lld K=%lld; K must be a multiple of 16)", (long long)groups,
              (long long)N, (long long)K);
  KW8_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15) == 0, KW8_ERR_UNSUPPORTED, "packed weights need 16-byte alignment");
  const int64_t FT = tiled_ftiles(N), KS = tiled_steps(K);
  const int64_t n = groups * FT * KS * 64;
  pack_kernel<<<pack_grid(n), 256, 0, stream>>>(q, groups, N, K, FT, KS, static_cast<uint4*>(out));
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_unpack(const void* tiled, int64_t groups, int64_t N, int64_t K, int8_t* q, cudaStream_t stream) {
  KW8_REQUIRE(tiled && q, KW8_ERR_INVALID_ARG, "null pointer");
  KW8_REQUIRE(groups >= 1 && N >= 1 && K >= 1 && K % 16 == 0, KW8_ERR_INVALID_ARG, "bad weight shape");
  KW8_REQUIRE((reinterpret_cast<uintptr_t>(tiled) & 15) == 0, KW8_ERR_UNSUPPORTED, "packed weights need 16-byte alignment");
  const int64_t FT = tiled_ftiles(N), KS = tiled_steps(K);
  const int64_t n = groups * FT * KS * 64;
  unpack_kernel<<<pack_grid(n), 256, 0, stream>>>(static_cast<const uint4*>(tiled), groups, N, K, FT, KS, q);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

}  // namespace kw8
