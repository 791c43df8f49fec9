// Expert-parallel MoE data movement over NVLink: peer-to-peer row copies
// into CUDA-IPC-mapped buffers of the other ranks (plain 16-byte stores;
// no TMA, no multicast).
//
// counts[s][e] (all ranks' kept rows per expert, from an all-gather) fixes
// every placement, so no host round trip is needed:
//   rank r owns experts [r*El, (r+1)*El);
//   its receive buffer is expert-major, source-major within an expert:
//     recv_pos(s, e, i) = Σ_{e' in r's experts, e' < e} Σ_s' counts[s'][e']
//                         + Σ_{s' < s} counts[s'][e] + i;
//   source s keeps its rows sorted by expert (the permutation's order):
//     src_pos(s, e, i) = Σ_{e' < e} counts[s][e'] + i.
#include "ep.cuh"

namespace kw8 {

namespace {

constexpr int kEpThreads = 256;

// dest_base[e] = recv_pos(src, e, 0) on e's owner for this source `src`
// (counts row s at counts + s * cstride).
__device__ void recv_bases(const int32_t* __restrict__ counts, int cstride, int world, int E, int El, int src,
                           int* dest_base) {
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int r0 = (e / El) * El;
    int base = 0;
    for (int e2 = r0; e2 < e; ++e2)
      for (int s = 0; s < world; ++s) base += counts[s * cstride + e2];
    for (int s = 0; s < src; ++s) base += counts[s * cstride + e];
    dest_base[e] = base;
  }
}

// Last index i in [0, n) with a[i] <= v (a non-decreasing, a[0] <= v).
__device__ __forceinline__ int upper_index(const int* a, int n, int v) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a[mid] <= v) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Row p of this rank's sorted order (expert e, i-th row of e) -> x[token]
// copied to recv_pos(rank, e, i) on e's owner.  A warp per row.
__global__ void __launch_bounds__(kEpThreads)
    ep_dispatch_kernel(const uint4* __restrict__ x, int vec, const int32_t* __restrict__ sorted_token,
                       const int32_t* __restrict__ offsets, const int32_t* __restrict__ counts, int world,
                       int rank, int E, int El, const uint64_t* __restrict__ peer_recv) {
  extern __shared__ int sh[];
  int* off = sh;            // [E+1] this rank's offsets
  int* dest = sh + E + 1;   // [E]
  for (int e = threadIdx.x; e <= E; e += blockDim.x) off[e] = offsets[e];
  recv_bases(counts, E, world, E, El, rank, dest);
  __syncthreads();
  const int rows = off[E];
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int p = blockIdx.x * wpb + (threadIdx.x >> 5); p < rows; p += gridDim.x * wpb) {
    const int e = upper_index(off, E + 1, p);
    const int pos = dest[e] + (p - off[e]);
    const uint4* src = x + static_cast<int64_t>(sorted_token[p]) * vec;
    uint4* dst = reinterpret_cast<uint4*>(peer_recv[e / El]) + static_cast<int64_t>(pos) * vec;
    for (int c = lane; c < vec; c += 32) dst[c] = src[c];
  }
  __threadfence_system();
}

// Local row q of this rank's receive layout (expert e, source s, i-th row)
// -> ys row copied to src_pos(s, e, i) on rank s.
__global__ void __launch_bounds__(kEpThreads)
    ep_return_kernel(const uint4* __restrict__ ys, int vec, const int32_t* __restrict__ counts, int world,
                     int rank, int E, int El, const uint64_t* __restrict__ peer_out) {
  extern __shared__ int sh[];
  int* start = sh;                 // [El*world + 1] local block starts, (expert, source) order
  int* dpos = sh + El * world + 1;  // [El*world]     src_pos(s, e, 0) on rank s
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int j = 0; j < El; ++j)
      for (int s = 0; s < world; ++s) {
        start[j * world + s] = acc;
        acc += counts[s * E + rank * El + j];
      }
    start[El * world] = acc;
  }
  for (int b = threadIdx.x; b < El * world; b += blockDim.x) {
    const int j = b / world, s = b % world, e = rank * El + j;
    int pos = 0;
    for (int e2 = 0; e2 < e; ++e2) pos += counts[s * E + e2];
    dpos[b] = pos;
  }
  __syncthreads();
  const int rows = start[El * world];
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int q = blockIdx.x * wpb + (threadIdx.x >> 5); q < rows; q += gridDim.x * wpb) {
    const int b = upper_index(start, El * world + 1, q);
    const int s = b % world;
    const uint4* src = ys + static_cast<int64_t>(q) * vec;
    uint4* dst = reinterpret_cast<uint4*>(peer_out[s]) + static_cast<int64_t>(dpos[b] + (q - start[b])) * vec;
    for (int c = lane; c < vec; c += 32) dst[c] = src[c];
  }
  __threadfence_system();
}

// Local experts' group offsets [El+1] of the receive layout.
__global__ void ep_local_offsets_kernel(const int32_t* __restrict__ counts, int cstride, int world, int rank,
                                        int El, int32_t* __restrict__ loc_off) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    int acc = 0;
    loc_off[0] = 0;
    for (int j = 0; j < El; ++j) {
      for (int s = 0; s < world; ++s) acc += counts[s * cstride + rank * El + j];
      loc_off[j + 1] = acc;
    }
  }
}

// ------------------------------------------------- group flags (peers) --
// Phase p of call `epoch` is done by rank r when flag word [p][r] of a
// rank's flags holds >= epoch.  Writers make their earlier stores visible
// system-wide first (fence), then store the flag with release semantics;
// waiters load it with acquire semantics, bounded by kWaitLimitNs.

__device__ __forceinline__ void flag_release(uint32_t* f, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t flag_acquire(const uint32_t* f) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}

// Epochs grow by one per call: v is at or past `epoch` when the unsigned
// difference is below half the range (robust to wrap-around).
__device__ __forceinline__ bool flag_reached(uint32_t v, uint32_t epoch) {
  return v - epoch < 0x80000000u;
}

__device__ bool flag_wait(const uint32_t* f, uint32_t epoch) {
  if (flag_reached(flag_acquire(f), epoch)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (flag_reached(flag_acquire(f), epoch)) return true;
    if ((i & 63u) == 0 && global_ns() - t0 > kWaitLimitNs) {
      report(KW8_ERR_DEVICE_TIMEOUT);
      return false;
    }
  }
}

// Signal (optionally) and wait for phase `phase` of `epoch`: lane r < world
// marks this rank's word at rank r, then waits for rank r's word here.
__global__ void ep_barrier_kernel(const uint64_t* __restrict__ flags, uint32_t* own_flags, int world,
                                  int rank, int phase, uint32_t epoch, int signal) {
  const int lane = threadIdx.x;
  if (signal && lane < world) {
    __threadfence_system();
    flag_release(reinterpret_cast<uint32_t*>(flags[lane]) + phase * world + rank, epoch);
  }
  if (lane < world) flag_wait(own_flags + phase * world + lane, epoch);
}

// This rank's per-expert row counts into every rank's counts[epoch & 1]
// (row `rank`), then phase 0 of the barrier: afterwards own counts[epoch &
// 1] holds every rank's counts.
__global__ void ep_counts_kernel(const int32_t* __restrict__ sizes, int E, const uint64_t* __restrict__ counts,
                                 const uint64_t* __restrict__ flags, uint32_t* own_flags, int world, int rank,
                                 uint32_t epoch) {
  const int parity = static_cast<int>(epoch & 1u);
  for (int p = 0; p < world; ++p) {
    int32_t* dst = reinterpret_cast<int32_t*>(counts[p]) + (static_cast<int64_t>(parity) * world + rank) * E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) dst[e] = sizes[e];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world) flag_release(reinterpret_cast<uint32_t*>(flags[threadIdx.x]) + rank, epoch);
  if (threadIdx.x < world) flag_wait(own_flags + threadIdx.x, epoch);
  __syncthreads();
}

// ------------------------------------------- one-shot partial-sum exchange --
// A group whose ranks each hold an fp32 partial [T][D] of the same output
// (tensor-parallel dense FFN, expert-parallel decode) sums it over NVLink:
// every rank stores its partial (the sum of its `splits` K-split slices)
// into slot [parity][rank] of every rank's exchange buffer, the group passes
// one flag phase, and every rank adds the world slots in rank order (the
// same order everywhere, so every rank gets the same bits).  parity =
// epoch & 1: a rank can start call e + 1 while a slower one still reads the
// slots of call e, but not call e + 2 (its phase waits for every rank's
// call e + 1), so two slot sets suffice.
// Call tag of a one-shot sum: the host's `epoch`, or (epoch == 0) the
// group's device-side counter at ctr (the last finished call) plus one, so
// that a call captured in a CUDA graph gets a new tag at every replay.
__device__ __forceinline__ uint32_t call_epoch(uint32_t epoch, const uint32_t* ctr) {
  return epoch != 0 ? epoch : *reinterpret_cast<const volatile uint32_t*>(ctr) + 1u;
}

// The whole sum is one cooperative launch (every CTA resident): each CTA
// pushes its share of this rank's partial into every rank's slot; the last
// CTA to arrive (counter at flags word 3 * world + 1) marks phase 1 of the
// call's tag at every rank; every CTA waits (bounded) for every rank's mark
// and adds its share of the world slots in rank order; the last CTA to
// leave (word 3 * world + 2) resets the counters and, with a device call
// count, stores the tag.
__global__ void __launch_bounds__(kEpThreads)
    ep_allreduce_kernel(const float4* __restrict__ part, int splits, int64_t split4, int64_t n4,
                        const uint64_t* __restrict__ peer_red, const float4* __restrict__ own_red,
                        const uint64_t* __restrict__ flags, uint32_t* own_flags, int world, int rank, int64_t slot4,
                        uint32_t epoch, uint2* __restrict__ out) {
  uint32_t* const ctr = own_flags + 3 * world;
  uint32_t* const arrive = ctr + 1;
  uint32_t* const depart = ctr + 2;
  __shared__ uint32_t e_sh;
  if (threadIdx.x == 0) e_sh = call_epoch(epoch, ctr);
  __syncthreads();
  const uint32_t e = e_sh;
  const int64_t par4 = static_cast<int64_t>(e & 1u) * world * slot4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4; i += stride) {
    float4 v = part[i];
    for (int sp = 1; sp < splits; ++sp) {
      const float4 b = part[sp * split4 + i];
      v.x += b.x; v.y += b.y; v.z += b.z; v.w += b.w;
    }
    for (int r = 0; r < world; ++r) reinterpret_cast<float4*>(peer_red[r])[par4 + rank * slot4 + i] = v;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(arrive, 1u) == gridDim.x - 1) {  // every CTA of this rank has pushed
      *reinterpret_cast<volatile uint32_t*>(arrive) = 0;
      __threadfence_system();
      for (int r = 0; r < world; ++r)
        flag_release(reinterpret_cast<uint32_t*>(flags[r]) + world + rank, e);
    }
    for (int r = 0; r < world; ++r) flag_wait(own_flags + world + r, e);
  }
  __syncthreads();
  const float4* slots = own_red + par4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4; i += stride) {
    float4 a = slots[i];
    for (int r = 1; r < world; ++r) {
      const float4 b = slots[r * slot4 + i];
      a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    }
    const __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y), hi = __floats2bfloat162_rn(a.z, a.w);
    out[i] = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
  }
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(depart, 1u) == gridDim.x - 1) {  // every CTA has read e and summed
    *reinterpret_cast<volatile uint32_t*>(depart) = 0;
    if (epoch == 0) *reinterpret_cast<volatile uint32_t*>(ctr) = e;
  }
}

int ep_grid_blocks(int64_t n) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + kEpThreads - 1) / kEpThreads, 148 * 8)));
}

int check_ep(int64_t D, int world, int rank, int64_t E) {
  KW8_REQUIRE(world >= 1 && world <= kEpMaxRanks && rank >= 0 && rank < world, KW8_ERR_INVALID_ARG,
              "bad rank %d of %d", rank, world);
  KW8_REQUIRE(E >= 1 && E <= 4096 && E % world == 0, KW8_ERR_INVALID_ARG,
              "%lld experts do not split over %d ranks", (long long)E, world);
  KW8_REQUIRE(D > 0 && D % 8 == 0, KW8_ERR_UNSUPPORTED, "D must be a multiple of 8");
  return KW8_OK;
}

}  // namespace

int launch_ep_dispatch(const void* x, int64_t max_rows, int64_t D, const int32_t* sorted_token,
                       const int32_t* offsets, const int32_t* counts, int world, int rank, int64_t E,
                       const uint64_t* peer_recv, cudaStream_t stream) {
  int rc = check_ep(D, world, rank, E);
  if (rc) return rc;
  if (max_rows <= 0) return KW8_OK;
  const int El = static_cast<int>(E / world);
  const size_t smem = (2 * E + 1) * sizeof(int);
  const int64_t blocks = std::min<int64_t>((max_rows + 7) / 8, 148 * 8);
  ep_dispatch_kernel<<<static_cast<int>(blocks), kEpThreads, smem, stream>>>(
      static_cast<const uint4*>(x), static_cast<int>(D / 8), sorted_token, offsets, counts, world, rank,
      static_cast<int>(E), El, peer_recv);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_ep_return(const void* ys, int64_t max_rows, int64_t D, const int32_t* counts, int world,
                     int rank, int64_t E, const uint64_t* peer_out, cudaStream_t stream) {
  int rc = check_ep(D, world, rank, E);
  if (rc) return rc;
  if (max_rows <= 0) return KW8_OK;
  const int El = static_cast<int>(E / world);
  const size_t smem = (2 * static_cast<size_t>(El) * world + 1) * sizeof(int);
  const int64_t blocks = std::min<int64_t>((max_rows + 7) / 8, 148 * 8);
  ep_return_kernel<<<static_cast<int>(blocks), kEpThreads, smem, stream>>>(
      static_cast<const uint4*>(ys), static_cast<int>(D / 8), counts, world, rank, static_cast<int>(E), El,
      peer_out);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_ep_local_offsets(const int32_t* counts, int world, int rank, int64_t E, int32_t* loc_off,
                            cudaStream_t stream, int64_t cstride) {
  int rc = check_ep(8, world, rank, E);
  if (rc) return rc;
  ep_local_offsets_kernel<<<1, 32, 0, stream>>>(counts, static_cast<int>(cstride > 0 ? cstride : E), world,
                                                rank, static_cast<int>(E / world), loc_off);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_ep_barrier(const uint64_t* flags, uint32_t* own_flags, int world, int rank, int phase,
                      uint32_t epoch, bool signal, cudaStream_t stream) {
  KW8_REQUIRE(world >= 1 && world <= kEpMaxRanks && rank >= 0 && rank < world && phase >= 0 &&
                  phase < 3,
              KW8_ERR_INVALID_ARG, "bad barrier args");
  ep_barrier_kernel<<<1, 32, 0, stream>>>(flags, own_flags, world, rank, phase, epoch, signal ? 1 : 0);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_ep_counts(const int32_t* sizes, int64_t E, const uint64_t* counts, const uint64_t* flags,
                     uint32_t* own_flags, int world, int rank, uint32_t epoch, cudaStream_t stream) {
  int rc = check_ep(8, world, rank, E);
  if (rc) return rc;
  ep_counts_kernel<<<1, 256, 0, stream>>>(sizes, static_cast<int>(E), counts, flags, own_flags, world, rank,
                                         epoch);
  KW8_CHECK_LAUNCH();
  return KW8_OK;
}

int launch_ep_allreduce(const float* part, int splits, int64_t split_stride, int64_t T, int64_t D,
                        const uint64_t* peer_red, float* own_red, int64_t red_rows, const uint64_t* flags,
                        uint32_t* own_flags, int world, int rank, uint32_t epoch, void* out, cudaStream_t stream) {
  KW8_REQUIRE(world >= 1 && world <= kEpMaxRanks && rank >= 0 && rank < world, KW8_ERR_INVALID_ARG,
              "bad rank %d of %d", rank, world);
  KW8_REQUIRE(T >= 0 && T <= red_rows && D % 4 == 0 && split_stride % 4 == 0 && splits >= 1,
              KW8_ERR_UNSUPPORTED, "partial sums of %lld rows exceed the exchange buffer (%lld rows)",
              (long long)T, (long long)red_rows);
  KW8_REQUIRE(((reinterpret_cast<uintptr_t>(part) | reinterpret_cast<uintptr_t>(own_red)) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(out) & 7) == 0,
              KW8_ERR_UNSUPPORTED, "partial sums need 16-byte aligned rows");
  // Every CTA of the launch must be resident at once (they wait for one
  // another): a cooperative launch of at most the co-resident CTAs.
  static int max_blocks[64] = {};
  int dev = 0;
  KW8_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) dev = 0;
  if (max_blocks[dev] == 0) {
    int per_sm = 0;
    KW8_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ep_allreduce_kernel, kEpThreads, 0));
    int sms = 0;
    KW8_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    KW8_REQUIRE(per_sm >= 1, KW8_ERR_UNSUPPORTED, "the exchange kernel does not fit an SM");
    max_blocks[dev] = per_sm * sms;
  }
  const int64_t n4 = T * D / 4;
  const int64_t slot4 = red_rows * D / 4;  // one rank's slot
  const int grid = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>({(n4 + kEpThreads - 1) / kEpThreads, 148 * 2, static_cast<int64_t>(max_blocks[dev])})));
  const float4* part4 = reinterpret_cast<const float4*>(part);
  int splits_a = splits;
  int64_t split4 = split_stride / 4;
  const float4* red4 = reinterpret_cast<const float4*>(own_red);
  uint2* out2 = static_cast<uint2*>(out);
  void* args[] = {&part4, &splits_a, &split4, const_cast<int64_t*>(&n4), &peer_red, &red4, &flags, &own_flags,
                  &world, &rank, const_cast<int64_t*>(&slot4), &epoch, &out2};
  KW8_CUDA_TRY(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(ep_allreduce_kernel), dim3(grid),
                                           dim3(kEpThreads), args, 0, stream));
  return KW8_OK;
}

}  // namespace kw8
