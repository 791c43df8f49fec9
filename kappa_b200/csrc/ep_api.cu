// C ABI of the expert-parallel row movement and its CUDA-IPC buffers.
#include <cstring>

#include "ep.cuh"

using namespace kw8;

extern "C" {

size_t kw8_ipc_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

int kw8_ipc_alloc(size_t bytes, void** ptr_out, void* handle_out) {
  KW8_API_BEGIN
  KW8_REQUIRE(ptr_out && handle_out && bytes > 0, KW8_ERR_INVALID_ARG, "bad ipc_alloc args");
  void* p = nullptr;
  KW8_CUDA_TRY(cudaMalloc(&p, bytes));
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(KW8_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *ptr_out = p;
  return KW8_OK;
}

int kw8_ipc_free(void* ptr) {
  KW8_API_BEGIN
  if (ptr) KW8_CUDA_TRY(cudaFree(ptr));
  return KW8_OK;
}

int kw8_ipc_open(const void* handle, void** ptr_out) {
  KW8_API_BEGIN
  KW8_REQUIRE(handle && ptr_out, KW8_ERR_INVALID_ARG, "bad ipc_open args");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  KW8_CUDA_TRY(cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess));
  return KW8_OK;
}

int kw8_ipc_close(void* ptr) {
  KW8_API_BEGIN
  if (ptr) KW8_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return KW8_OK;
}

int kw8_ep_dispatch(const void* x, int64_t max_rows, int64_t D, const int32_t* sorted_token,
                    const int32_t* group_offsets, const int32_t* counts, int32_t world, int32_t rank,
                    int64_t E, const uint64_t* peer_recv, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(x && sorted_token && group_offsets && counts && peer_recv, KW8_ERR_INVALID_ARG,
              "null pointer");
  return launch_ep_dispatch(x, max_rows, D, sorted_token, group_offsets, counts, world, rank, E,
                            peer_recv, static_cast<cudaStream_t>(stream));
}

int kw8_ep_return(const void* ys, int64_t max_rows, int64_t D, const int32_t* counts, int32_t world,
                  int32_t rank, int64_t E, const uint64_t* peer_out, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(ys && counts && peer_out, KW8_ERR_INVALID_ARG, "null pointer");
  return launch_ep_return(ys, max_rows, D, counts, world, rank, E, peer_out,
                          static_cast<cudaStream_t>(stream));
}

int kw8_ep_local_offsets(const int32_t* counts, int32_t world, int32_t rank, int64_t E,
                         int32_t* local_offsets, kw8_stream_t stream) {
  KW8_API_BEGIN
  KW8_REQUIRE(counts && local_offsets, KW8_ERR_INVALID_ARG, "null pointer");
  return launch_ep_local_offsets(counts, world, rank, E, local_offsets,
                                 static_cast<cudaStream_t>(stream));
}

}  // extern "C"
