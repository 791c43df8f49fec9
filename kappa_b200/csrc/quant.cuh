// W8 quantisation / dequantisation kernels (see quant.cu).
#pragma once

#include "common.cuh"

namespace kw8 {

size_t quantize_workspace_size(int64_t outer, int64_t N);
int launch_quantize(const void* w, int w_dtype, int64_t outer, int64_t K, int64_t N, int64_t so,
                    int64_t sk, int64_t sn, int per_channel, int scale_dtype, int8_t* q,
                    void* scale_out, void* ws, size_t ws_bytes, cudaStream_t stream);
int launch_dequantize(const kw8_weight& w, int64_t groups, int64_t N, int64_t K, int out_dtype,
                      void* out, cudaStream_t stream);
// Quantised embedding rows: out[i] = dequant(table[tokens[i]]) ([V][D] int8).
int launch_embed_gather(const int32_t* tokens, int64_t n, const kw8_weight& table, int64_t V,
                        int64_t D, int out_dtype, void* out, cudaStream_t stream);

}  // namespace kw8
