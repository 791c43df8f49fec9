// kw8_moe_ffn_noalloc: the MoE layer for callers that cannot allocate device
// memory where they call it.
//
// Some callers have no way to hand this library a workspace: a custom-call
// handler that is given only its input and output buffers and no scratch
// allocator, or a host program whose device memory is owned by another
// allocator it cannot reach from the call site (and where calling
// cudaMalloc itself would fragment or exceed that allocator's budget).  For
// them the scratch lives here, in a fixed array that every GPU loading the
// library holds until the process exits.
#include <mutex>

#include "common.cuh"

extern "C" size_t kw8_moe_ffn_workspace_size(int64_t T, int64_t D, int64_t I, int64_t E,
                                             int32_t k);
extern "C" int kw8_moe_ffn(const void* x, int64_t T, int64_t D, int64_t I, int64_t E, int32_t k,
                           int64_t capacity, kw8_weight router, kw8_weight gate, kw8_weight up,
                           kw8_weight down, void* out, void* workspace, size_t workspace_bytes,
                           kw8_stream_t stream);

namespace kw8 {
void clear_error();

namespace {

// Largest scratch a call may use: 16 MiB per GPU.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

// The scratch itself.  In host code this name is only a stand-in for the
// device array; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};
void* g_noalloc_ctx[kMaxDevices] = {};  // the context the address was looked up in

// The calling thread's current CUDA context (cuCtxGetCurrent, found through
// the runtime's driver entry point), or null if it cannot be read.
void* current_context() {
  using GetCurrentFn = int (*)(void**);
  static GetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetCurrentFn>(p);
  });
  void* ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// Device address of the scratch on the current device, looked up (with
// that device current) once per device and context and cached: a device
// reset or another context on the device gets a fresh lookup.
int noalloc_scratch(void** addr) {
  int dev = 0;
  KW8_CUDA_TRY(cudaGetDevice(&dev));
  KW8_REQUIRE(dev >= 0 && dev < kMaxDevices, KW8_ERR_UNSUPPORTED, "device %d out of range", dev);
  void* ctx = current_context();
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr || ctx == nullptr || ctx != g_noalloc_ctx[dev]) {
    void* p = nullptr;
    KW8_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    KW8_REQUIRE(p != nullptr, KW8_ERR_CUDA, "scratch address lookup returned null");
    g_noalloc_addr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *addr = g_noalloc_addr[dev];
  return KW8_OK;
}

}  // namespace
}  // namespace kw8

extern "C" int kw8_moe_ffn_noalloc(const void* x, int64_t T, int64_t D, int64_t I, int64_t E,
                                   int32_t k, int64_t capacity, kw8_weight router,
                                   kw8_weight gate, kw8_weight up, kw8_weight down, void* out,
                                   kw8_stream_t stream) {
  kw8::clear_error();
  if (T < 0 || D <= 0 || I <= 0 || E <= 0 || k < 1)
    return kw8::fail(KW8_ERR_INVALID_ARG, "bad shape (T=%lld D=%lld I=%lld E=%lld k=%d)",
                     (long long)T, (long long)D, (long long)I, (long long)E, k);
  const size_t need = kw8_moe_ffn_workspace_size(T, D, I, E, k);
  if (need > kw8::kNoAllocScratchBytes)
    return kw8::fail(KW8_ERR_WORKSPACE,
                     "kw8_moe_ffn_noalloc: these shapes need %zu bytes of scratch, more than the "
                     "%zu bytes built into the library; call kw8_moe_ffn with a workspace instead",
                     need, kw8::kNoAllocScratchBytes);
  void* scratch = nullptr;
  const int rc = kw8::noalloc_scratch(&scratch);
  if (rc) return rc;
  // Nothing in the scratch has to start at zero: kw8_moe_ffn writes every
  // buffer before reading it and clears its fp32 combine buffer itself.
  return kw8_moe_ffn(x, T, D, I, E, k, capacity, router, gate, up, down, out, scratch,
                     kw8::kNoAllocScratchBytes, stream);
}
