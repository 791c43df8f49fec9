// Single translation unit of libkappa_w8.so: the parts share one device
// status word and are compiled together so no relocatable device code is
// needed.
#include "host.cu"
#include "pack.cu"
#include "quant.cu"
#include "gemm_tc.cu"
#include "gemm_tc2.cu"
#include "gemm_stream.cu"
#include "moe.cu"
#include "norm.cu"
#include "api.cu"
#include "noalloc.cu"
#include "ep.cu"
#include "ep_dedup.cu"
#include "ep_api.cu"
