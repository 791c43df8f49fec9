// Host-side support: per-thread error strings, the device status word read
// back, and TMA descriptor encoding (cuTensorMapEncodeTiled reached through
// the runtime's driver entry point, so the library needs no -lcuda).
#include <cstdarg>
#include <mutex>

#include "common.cuh"

namespace kw8 {

namespace {
thread_local std::string t_last_error;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
}  // namespace

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
}

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

const char* last_error() { return t_last_error.c_str(); }
void clear_error() { t_last_error.clear(); }

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype, int esize,
                 uint64_t rows, uint64_t cols, uint64_t pitch_bytes, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  KW8_REQUIRE(fn != nullptr, KW8_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  KW8_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0, KW8_ERR_UNSUPPORTED,
              "TMA base address must be 16-byte aligned");
  KW8_REQUIRE(pitch_bytes % 16 == 0, KW8_ERR_UNSUPPORTED, "TMA row pitch must be a multiple of 16");
  KW8_REQUIRE((static_cast<uint64_t>(box_cols) * esize) % 16 == 0 && box_rows >= 1 &&
                  box_rows <= 256 && box_cols <= 256,
              KW8_ERR_INVALID_ARG, "bad TMA box");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {pitch_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  KW8_REQUIRE(r == CUDA_SUCCESS, KW8_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return KW8_OK;
}

int make_tmap_tiled(CUtensorMap* map, const void* base, uint64_t tile_rows, uint64_t steps,
                    uint32_t box_tiles) {
  EncodeTiledFn fn = encode_fn();
  KW8_REQUIRE(fn != nullptr, KW8_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  KW8_REQUIRE((reinterpret_cast<uintptr_t>(base) & 15) == 0, KW8_ERR_UNSUPPORTED,
              "TMA base address must be 16-byte aligned");
  KW8_REQUIRE(box_tiles >= 1 && box_tiles <= 256 && steps % 2 == 0 && tile_rows >= 1, KW8_ERR_INVALID_ARG,
              "bad tiled TMA box");
  // [tile_rows][steps * 4][256 bytes]; a box is [box_tiles][8][256]: the
  // two 1 KB blocks of one 128-k stage of box_tiles feature tiles.
  const cuuint64_t dims[3] = {256, steps * 4, tile_rows};
  const cuuint64_t strides[2] = {256, steps * 1024};
  const cuuint32_t box[3] = {256, 8, box_tiles};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  KW8_REQUIRE(r == CUDA_SUCCESS, KW8_ERR_CUDA, "cuTensorMapEncodeTiled (tiled weights) failed (%d)", (int)r);
  return KW8_OK;
}

int read_device_status(int32_t* out, cudaStream_t stream) {
  KW8_REQUIRE(out != nullptr, KW8_ERR_INVALID_ARG, "null status pointer");
  KW8_CUDA_TRY(cudaStreamSynchronize(stream));
  int v = 0;
  KW8_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)));
  const int zero = 0;
  KW8_CUDA_TRY(cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)));
  *out = v;
  return KW8_OK;
}

}  // namespace kw8
