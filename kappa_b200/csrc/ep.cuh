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
// counts rows are cstride ints apart (0: E).
int launch_ep_local_offsets(const int32_t* counts, int world, int rank, int64_t E, int32_t* loc_off,
                            cudaStream_t stream, int64_t cstride = 0);
// Group flags (kw8_ep_peers): phase `phase` of `epoch`, signalled first
// when `signal`; and the counts exchange (phase 0).
int launch_ep_barrier(const uint64_t* flags, uint32_t* own_flags, int world, int rank, int phase,
                      uint32_t epoch, bool signal, cudaStream_t stream);
int launch_ep_counts(const int32_t* sizes, int64_t E, const uint64_t* counts, const uint64_t* flags,
                     uint32_t* own_flags, int world, int rank, uint32_t epoch, cudaStream_t stream);

// One-shot sum of fp32 partials [T][D] over the group (see ep.cu), one
// cooperative launch: push (the sum of `splits` slices split_stride floats
// apart) into every rank's exchange buffer [2][world][red_rows][D], flag
// phase 1 of `epoch`, then out = bf16(sum over ranks in rank order).  The
// flags buffer holds 3 * world + 3 words (call count, two CTA counters).
int launch_ep_allreduce(const float* part, int splits, int64_t split_stride, int64_t T, int64_t D,
                        const uint64_t* peer_red, float* own_red, int64_t red_rows, const uint64_t* flags,
                        uint32_t* own_flags, int world, int rank, uint32_t epoch, void* out, cudaStream_t stream);

// Token-deduplicated step (ep_dedup.cu).
int launch_ep_slots(const int32_t* idx, const int32_t* inv_pos, int64_t T, int k, int64_t E, int world,
                    int32_t* tok_slot, int32_t* u_cnt, cudaStream_t stream);
int launch_ep_counts2(const int32_t* sizes, const int32_t* u_cnt, int64_t E, const uint64_t* counts,
                      const uint64_t* flags, uint32_t* own_flags, int world, int rank, uint32_t epoch,
                      cudaStream_t stream);
int launch_ep_dispatch2(const void* x, int64_t T, int k, int64_t D, const int32_t* sorted_token,
                        const int32_t* offsets, const float* sorted_w, const int32_t* tok_slot,
                        const int32_t* counts, int world, int rank, int64_t E, int64_t pair_cap,
                        const uint64_t* peer_rows, const uint64_t* peer_meta, cudaStream_t stream);
int launch_ep_gather2(const void* rows, const int32_t* meta, const int32_t* loc_off, int64_t El,
                      const int32_t* counts, int world, int rank, int64_t E, int64_t D, int64_t max_pairs,
                      void* xs, float* part, cudaStream_t stream);
int launch_ep_return2(const float* part, int64_t D, const int32_t* counts, int world, int rank, int64_t E,
                      int64_t max_tokens, const uint64_t* peer_ret, int ret_format, cudaStream_t stream);
int launch_ep_final2(const void* ret, const int32_t* tok_slot, int64_t T, int world, int64_t max_tokens,
                     int64_t D, int ret_format, void* out, cudaStream_t stream);

}  // namespace kw8
