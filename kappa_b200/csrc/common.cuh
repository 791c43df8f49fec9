// Shared device/host helpers for the kappa_w8 kernels (sm_100a only).
//
// PTX wrappers for mbarrier, TMA (cp.async.bulk.tensor, never with cluster
// multicast) and the 5th-generation tensor core (tcgen05.*), bounded
// waits that give up instead of hanging, and the per-thread host error
// string behind kw8_last_error().
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <string>

#include "../../include/kappa_w8.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "kappa_w8 kernels target sm_100a only"
#endif

namespace kw8 {

// ------------------------------------------------------------ host errors --

void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
#define KW8_CUDA_TRY(expr)                                                   \
  do {                                                                       \
    cudaError_t e__ = (expr);                                                \
    if (e__ != cudaSuccess)                                                  \
      return ::kw8::fail(KW8_ERR_CUDA, "%s: %s (%s:%d)", #expr,              \
                         cudaGetErrorString(e__), __FILE__, __LINE__);       \
  } while (0)
#define KW8_CHECK_LAUNCH() KW8_CUDA_TRY(cudaGetLastError())
#define KW8_REQUIRE(cond, code, ...)                                         \
  do {                                                                       \
    if (!(cond)) return ::kw8::fail((code), __VA_ARGS__);                    \
  } while (0)

// Device status word: kernels write a kw8_status here (first writer wins)
// when a bounded wait runs out or an index check fails.  Defined here: the
// library is one translation unit (kappa_w8.cu).
__device__ int g_device_status = 0;

__device__ __forceinline__ void report(int code) {
  atomicCAS(&g_device_status, 0, code);
}

// Upper bound on any single wait inside a kernel.  Kernels of this library
// finish in milliseconds; a wait this long means a broken pipeline, and the
// kernel then stops waiting, records KW8_ERR_DEVICE_TIMEOUT and exits.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Process-wide option (kw8_set_option 4): time the phases of
// kw8_moe_ffn_ep with CUDA events (read back with kw8_ep_phase_times).
inline std::atomic<int> g_opt_ep_timing{0};

// ----------------------------------------------------------- small utils --

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

__device__ __forceinline__ float load_scale(const void* p, int dtype, int64_t i) {
  if (dtype == KW8_DT_F32) return __ldg(static_cast<const float*>(p) + i);
  const uint16_t* b = static_cast<const uint16_t*>(p);
  return bf16_bits_to_f32(__ldg(b + i));
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// int8 x4 (one 32-bit word, byte 0 = lowest k) -> two bf16x2 words, exact,
// in two instructions per element.  For a byte b (two's complement q) the
// 16-bit lane t = 0x43:b is formed with one byte_perm; then
//   x = t & 0xFF7F  is bf16 128 + (b & 0x7F)
//   c = t & 0xFF80  is bf16 128 (b >= 0) or 256 (b < 0, 0x4380)
// and x - c = q: 128 + q - 128 for q >= 0, 128 + (q + 128) - 256 for q < 0.
// The bf16 subtraction is exact (c/2 <= x <= 2c and q is representable).
__device__ __forceinline__ void i8x4_to_bf16x4(uint32_t w, uint32_t& lo,
                                               uint32_t& hi) {
  const uint32_t t0 = __byte_perm(w, 0x43434343u, 0x4140);  // 43:b1:43:b0
  const uint32_t t1 = __byte_perm(w, 0x43434343u, 0x4342);  // 43:b3:43:b2
  lo = bf16x2_sub(t0 & 0xFF7FFF7Fu, t0 & 0xFF80FF80u);
  hi = bf16x2_sub(t1 & 0xFF7FFF7Fu, t1 & 0xFF80FF80u);
}

__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float gelu_tanh_f(float x) {
  // jax.nn.gelu(approximate=True): 0.5 x (1 + tanh(sqrt(2/pi)(x + 0.044715 x^3))),
  // with the hardware tanh approximation (relative error < 2^-10).
  const float c = 0.7978845608028654f;
  const float inner = c * (x + 0.044715f * x * x * x);
  return 0.5f * x * (1.0f + tanh_approx(inner));
}

__device__ __forceinline__ float silu_f(float x) {
  // jax.nn.silu: x * sigmoid(x) = x / (1 + e^-x), fast exp and divide.
  return __fdividef(x, 1.0f + __expf(-x));
}

// --------------------------------------------------------------- mbarrier --

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with parity `parity` to complete.  Returns false (and
// records KW8_ERR_DEVICE_TIMEOUT, or sees that another warp did) if it does
// not complete within kWaitLimitNs, or if *abort becomes non-zero.  With
// abort == nullptr only the time limit applies.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (abort && *abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        if (abort) *abort = 1;
        report(KW8_ERR_DEVICE_TIMEOUT);
        return false;
      }
    }
  }
}

// ------------------------------------------------ CTA pairs (clusters) --

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the same shared-memory location in CTA `rank`
// of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}

// Arrive (release at cluster scope) on an mbarrier given by its
// shared::cluster address (this CTA's or the peer's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// mbar_wait for a barrier that other CTAs of the cluster arrive on
// (acquire at cluster scope); same bounds as mbar_wait.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (abort && *abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        if (abort) *abort = 1;
        report(KW8_ERR_DEVICE_TIMEOUT);
        return false;
      }
    }
  }
}

// Every thread of both CTAs of the cluster: arrive and wait.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// -------------------------------------------------------------------- TMA --

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m))
               : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory (no multicast).
__device__ __forceinline__ void tma_load_2d(void* smem_dst,
                                            const CUtensorMap* map,
                                            uint64_t* bar, int32_t c0,
                                            int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1),
      "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled TMA load (no multicast): box at coordinates (c0, c1, c2).
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- tcgen05 --

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Warp-wide: allocate `ncols` TMEM columns; the base address is written to
// *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst_smem)),
      "r"(ncols)
      : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}

// D[tmem] (+)= A[tmem] x B[smem]ᵀ, kind::f16 (bf16 operands, fp32 accumulate).
__device__ __forceinline__ void mma_ts_bf16(uint32_t d_tmem, uint32_t a_tmem,
                                            uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 op this thread issued has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_u32(bar))
      : "memory");
}

// Warp-wide, in both CTAs of a pair (the same warp of each): allocate
// `ncols` TMEM columns at the same address in both.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst_smem)),
      "r"(ncols)
      : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D[tmem] (+)= A[tmem] x B[smem]^T over a CTA pair (M = 256: each CTA's
// TMEM holds 128 rows of A and of D, each CTA's shared memory N/2 rows of
// B at the same address), kind::f16.  Issued by one thread of CTA 0.
__device__ __forceinline__ void mma_ts_bf16_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` (same shared-memory offset) in both CTAs of the pair once
// every tcgen05 op this thread issued has completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// Instruction descriptor, kind::f16: A = B = bf16 (both K-major), D = f32.
__device__ __forceinline__ uint32_t idesc_bf16_f32(uint32_t M, uint32_t N) {
  return (1u << 4)            // D format: f32
         | (1u << 7)          // A format: bf16
         | (1u << 10)         // B format: bf16
         | ((N >> 3) << 17)   // N / 8
         | ((M >> 4) << 24);  // M / 16
}

// Shared-memory matrix descriptor for a K-major operand staged by TMA with
// 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart (SBO).
__device__ __forceinline__ uint64_t smem_desc_kmajor_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address
  d |= static_cast<uint64_t>(1) << 16;                  // LBO (unused) = 16 B
  d |= static_cast<uint64_t>(1024 >> 4) << 32;          // SBO = 1024 B
  d |= static_cast<uint64_t>(1) << 46;                  // descriptor version
  d |= static_cast<uint64_t>(2) << 61;                  // SWIZZLE_128B
  return d;
}

#define KW8_TMEM_ST_X32(taddr, v)                                              \
  asm volatile(                                                                \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, " \
      "%7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, "    \
      "%21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(    \
          taddr),                                                              \
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),       \
      "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]),     \
      "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), \
      "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), \
      "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), \
      "r"(v[30]), "r"(v[31])                                                   \
      : "memory")

#define KW8_TMEM_ST_X16(taddr, v)                                              \
  asm volatile(                                                                \
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, " \
      "%7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),          \
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),       \
      "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]),     \
      "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])                           \
      : "memory")

#define KW8_TMEM_LD_X32(taddr, v)                                              \
  asm volatile(                                                                \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, "   \
      "%7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, "    \
      "%21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"         \
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]),           \
        "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]),           \
        "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),      \
        "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),      \
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),      \
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),      \
        "=r"(v[30]), "=r"(v[31])                                               \
      : "r"(taddr)                                                             \
      : "memory")

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------ host-side TMA maps --

// Encodes a 2-D row-major tensor map ([rows][cols], element size `esize`,
// row pitch `pitch_bytes`) with box (box_cols, box_rows).  Returns KW8_OK or
// a kw8_status (with kw8_last_error set).
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                 int esize, uint64_t rows, uint64_t cols, uint64_t pitch_bytes,
                 uint32_t box_cols, uint32_t box_rows,
                 CUtensorMapSwizzle swizzle);

// Tensor map of a pre-packed (tiled) int8 weight with `tile_rows` feature
// tiles of `steps` 1 KB blocks each, viewed as [tile_rows][steps * 4][256 B];
// box: 2 steps (one 128-k stage) of `box_tiles` feature tiles.
int make_tmap_tiled(CUtensorMap* map, const void* base, uint64_t tile_rows, uint64_t steps,
                    uint32_t box_tiles);

}  // namespace kw8
