// Expert-parallel row movement over NVLink (see ep.cu).
#pragma once

#include "common.cuh"

namespace kw8 {

constexpr int kEpMaxRanks = 8;

int launch_ep_dispatch(const void* x, int64_t max_rows, int64_t D, const int32_t* sorted_token,
                       const int32_t* offsets, const int32_t* counts, int world, int rank, int64_t E,
                       const uint64_t* peer_recv, cudaStream_t stream);
int launch_ep_return(const void* ys, int64_t max_rows, int64_t D, const int32_t* counts, int world,
                     int rank, int64_t E, const uint64_t* peer_out, cudaStream_t stream);
int launch_ep_local_offsets(const int32_t* counts, int world, int rank, int64_t E, int32_t* loc_off,
                            cudaStream_t stream);
// Group flags (kw8_ep_peers): phase `phase` of `epoch`, signalled first
// when `signal`; and the counts exchange (phase 0).
int launch_ep_barrier(const uint64_t* flags, uint32_t* own_flags, int world, int rank, int phase,
                      uint32_t epoch, bool signal, cudaStream_t stream);
int launch_ep_counts(const int32_t* sizes, int64_t E, const uint64_t* counts, const uint64_t* flags,
                     uint32_t* own_flags, int world, int rank, uint32_t epoch, cudaStream_t stream);

}  // namespace kw8
