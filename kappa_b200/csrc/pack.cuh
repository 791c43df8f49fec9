// Pre-packed ("tiled") W8 weight layout (see pack.cu).
#pragma once

#include "common.cuh"

namespace kw8 {

constexpr int kTiledRows = 16;     // rows of a feature tile
constexpr int kTiledStepK = 64;    // k of a step
constexpr int kTiledBlock = 1024;  // bytes of a (feature tile, step) block

inline int64_t tiled_ftiles(int64_t N) { return (N + kTiledRows - 1) / kTiledRows; }
// Steps of 64 k with K padded to a multiple of 128 (whole tensor-core stages).
inline int64_t tiled_steps(int64_t K) { return (K + 127) / 128 * 2; }
inline int64_t tiled_bytes(int64_t groups, int64_t N, int64_t K) {
  return groups * tiled_ftiles(N) * tiled_steps(K) * kTiledBlock;
}

// K-major [groups][N][K] int8 -> tiled (tiled_bytes(groups, N, K) bytes).
int launch_pack(const int8_t* q, int64_t groups, int64_t N, int64_t K, void* out, cudaStream_t stream);
// Tiled -> K-major [groups][N][K] int8.
int launch_unpack(const void* tiled, int64_t groups, int64_t N, int64_t K, int8_t* q, cudaStream_t stream);

}  // namespace kw8
