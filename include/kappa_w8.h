/*
 * kappa_w8.h — C ABI of the B200 (sm_100a) W8 fake-quant feed-forward path.
 *
 * This library replaces the int8-weight ("W8") feed-forward hot path of the
 * JAX inference library kappa (baricev/kappa, version 0.0.1).  kappa has no
 * FFI layer of its own: its boundary is a set of pure Python functions.  Each
 * entry point below names the kappa function (file:line, paths relative to
 * the kappa project root) whose behaviour it reproduces.
 *
 * Conventions shared by every entry point
 *   - Pointers are CUDA device pointers unless stated otherwise; the caller
 *     owns every buffer.  The library never allocates on these paths: scratch
 *     memory comes from the caller through (workspace, workspace_bytes), and
 *     each *_workspace_size() query states how much is needed.
 *   - Work is enqueued on `stream` (a cudaStream_t) and is stream ordered.
 *     Nothing synchronises the host except kw8_device_status().
 *   - Return value: KW8_OK (0) or a negative kw8_status.  A human readable
 *     message for the last failure on the calling thread is returned by
 *     kw8_last_error().
 *   - Activations are bf16, row major [tokens][features].
 *   - W8 weights are int8 stored K-major ("contraction axis innermost"):
 *     a weight that maps K inputs to N outputs is [N][K] int8, row stride K.
 *     Stacked expert weights are [E][N][K].  kappa's logical layouts
 *     ([E, D, I] for gate/up, [E, I, D] for down, [2, H, D] for the Gemma
 *     gating einsum) are views of these buffers; the Python layer
 *     (kappa_b200) keeps kappa's logical shapes.
 *   - K must be a multiple of 16 (row starts stay 16-byte aligned, which the
 *     TMA engine requires); other shapes return KW8_ERR_UNSUPPORTED.
 */
#ifndef KAPPA_W8_H_
#define KAPPA_W8_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* kw8_stream_t; /* identical to cudaStream_t */

typedef enum kw8_status {
  KW8_OK = 0,
  KW8_ERR_INVALID_ARG = -1,    /* null pointer, bad shape, bad enum        */
  KW8_ERR_UNSUPPORTED = -2,    /* shape outside what the kernels handle    */
  KW8_ERR_CUDA = -3,           /* a CUDA runtime / driver call failed      */
  KW8_ERR_WORKSPACE = -4,      /* workspace missing or too small           */
  KW8_ERR_DEVICE_TIMEOUT = -5, /* a kernel's bounded wait ran out          */
} kw8_status;

typedef enum kw8_dtype { KW8_DT_F32 = 0, KW8_DT_BF16 = 1 } kw8_dtype;

typedef enum kw8_act {
  KW8_ACT_GELU_TANH = 0, /* jax.nn.gelu default (approximate=True)          */
  KW8_ACT_SILU = 1,      /* jax.nn.silu                                      */
} kw8_act;

/* RMSNorm flavour: out = x * rsqrt(mean(x^2) + eps) * g with
 * g = 1 + scale (Gemma3, kappa/gemma3/norms.py:8-13) or
 * g = scale     (Qwen3,  kappa/qwen3/norms.py:10-16).                       */
typedef enum kw8_norm_kind { KW8_NORM_GEMMA = 0, KW8_NORM_QWEN = 1 } kw8_norm_kind;

/* Storage of the int8 values of a W8 weight.
 *   KW8_LAYOUT_KMAJOR: [groups][N][K], K contiguous (row stride K).
 *   KW8_LAYOUT_TILED : pre-packed by kw8_pack_weight:
 *     [groups][ceil(N/16)][2*ceil(K/128)][1024 bytes]; block (g, f, s)
 *     holds rows 16f..16f+15 and k = 64s..64s+63, the 16 k of chunk c
 *     (c = 0..3) of row 16f + 8h + r (h = 0..1, r = 0..7) at byte
 *     512h + 16(8c + r); zeros past N and K.  Each kernel reads it in
 *     whole contiguous pieces (512 B per warp load in the decode kernel,
 *     one 16 KB box per tensor-core stage).                               */
typedef enum kw8_layout { KW8_LAYOUT_KMAJOR = 0, KW8_LAYOUT_TILED = 1 } kw8_layout;

/* One W8 weight: int8 values plus either one scale for the whole tensor
 * (kappa's Q8Weight, kappa/qwen3/quant.py:15-19) or one scale per output
 * channel (per expert when stacked): [groups][N] scales.                    */
typedef struct kw8_weight {
  const int8_t* q;     /* the int8 values in `layout`                       */
  const void* scale;   /* 1 value, or [groups][N] values                    */
  int32_t scale_dtype; /* kw8_dtype of `scale`                              */
  int32_t per_channel; /* 0: one scale; 1: [groups][N] scales               */
  int32_t layout;      /* kw8_layout of `q`                                 */
  int32_t reserved;    /* 0                                                 */
} kw8_weight;

/* ---------------------------------------------------------------- misc -- */

/* Message for the last failing call on this host thread ("" if none).      */
const char* kw8_last_error(void);

/* ABI version of this library (bumped on any signature change).            */
int32_t kw8_abi_version(void);

/* Reads and clears the device-side status word that kernels set when a
 * bounded wait runs out (KW8_ERR_DEVICE_TIMEOUT) or a kernel-side check
 * fails (KW8_ERR_INVALID_ARG: an expert id out of range, e.g. a token whose
 * router logits are NaN; its routed entries are dropped and its output row
 * is zero).  Synchronises `stream`.  *status_out receives 0 or a kw8_status. */
int kw8_device_status(int32_t* status_out, kw8_stream_t stream);

/* Tuning and testing knobs, process wide; no kappa counterpart (kappa
 * leaves kernel choice to XLA).
 *   option 0 (GEMM path): 0 automatic, 1 tensor-core GEMM, 2 weight-
 *            streaming GEMM (the decode kernel: few rows per group);
 *   option 1 (token tile of the tensor-core GEMM): 0 automatic, or a
 *            multiple of 16 in [16, 256];
 *   option 2 (MoE combine): 0 the fused fp32 combine of the down GEMM's
 *            epilogue (its additions run in arrival order), 1 a fixed
 *            order: the expert outputs are stored as bf16 rows and every
 *            token's k rows are summed in slot order (bit-identical runs);
 *   option 3 (tensor-core GEMM over SM pairs, cta_group::2 with M = 256):
 *            0 automatic (the one-CTA kernel, faster where measured),
 *            1 never, 2 for every launch whose tile allows it;
 *   option 4 (phase timing of kw8_moe_ffn_ep's deduplicated step): 1
 *            records CUDA events at its phase boundaries (see
 *            kw8_ep_phase_times), 0 none.                                    */
int kw8_set_option(int32_t option, int64_t value);

/* ------------------------------------------------------- quantisation -- */

/* quantize_weight (kappa/qwen3/quant.py:41-48), per tensor or per channel.
 *   w        : f32 or bf16 weight with logical shape [outer][K][N] given by
 *              element strides (stride_outer, stride_k, stride_n), so both
 *              [.., K, N] (N contiguous) and [.., N, K] (K contiguous)
 *              inputs are accepted without a copy.
 *   per_channel = 0 : amax over the whole tensor (kappa's behaviour);
 *   per_channel = 1 : amax over K for every (outer, n) output channel.
 *   scale = max(amax / 127, FLT_MIN) in fp32 (IEEE division);
 *   q     = clip(round_half_even(w / scale), -128, 127)  using the fp32 scale;
 *   stored scale = scale rounded (RNE) to scale_dtype.
 *   q_out     : [outer][N][K] int8 (K-major).
 *   scale_out : 1 value (per tensor) or [outer][N] values, scale_dtype.
 *   workspace : >= kw8_quantize_workspace_size(outer, N) bytes, 4-byte
 *               aligned (per-channel absmax scratch).                       */
size_t kw8_quantize_workspace_size(int64_t outer, int64_t N);
int kw8_quantize(const void* w, int32_t w_dtype, int64_t outer, int64_t K,
                 int64_t N, int64_t stride_outer, int64_t stride_k,
                 int64_t stride_n, int32_t per_channel, int32_t scale_dtype,
                 int8_t* q_out, void* scale_out, void* workspace,
                 size_t workspace_bytes, kw8_stream_t stream);

/* to_compute_dtype (kappa/qwen3/quant.py:34-38) for a W8 weight:
 * out[g][n][k] = dtype(q[g][n][k]) * dtype(scale)  (one rounding per
 * product, as kappa's `values.astype(dt) * scale.astype(dt)`).
 * out is [groups][N][K] in out_dtype.                                       */
int kw8_dequantize(kw8_weight w, int64_t groups, int64_t N, int64_t K,
                   int32_t out_dtype, void* out, kw8_stream_t stream);

/* Pre-packed weights: the load-time step that kappa's quantize_qwen3_params
 * (kappa/qwen3/weights.py:143-170) would end with, so that every kernel
 * reads whole contiguous pieces of the weights.  q [groups][N][K] int8
 * (K % 16 == 0) -> tiled (kw8_packed_weight_bytes bytes, 16-byte aligned),
 * and back.  The values are the same bits; scales are unchanged.          */
size_t kw8_packed_weight_bytes(int64_t groups, int64_t N, int64_t K);
int kw8_pack_weight(const int8_t* q, int64_t groups, int64_t N, int64_t K, void* tiled,
                    kw8_stream_t stream);
int kw8_unpack_weight(const void* tiled, int64_t groups, int64_t N, int64_t K, int8_t* q,
                      kw8_stream_t stream);

/* ----------------------------------------------------------- dense FFN -- */

/* Gated dense FFN:
 *   Gemma3 feed_forward (kappa/gemma3/ffn.py:10-26) with act = GELU_TANH and
 *     gate = gating[0], up = gating[1] ([H][D] each, transpose_gating_einsum
 *     layout), down = linear viewed K-major ([D][H]);
 *   Qwen3 swiglu_ffn (kappa/qwen3/ffn.py:12-22) with act = SILU.
 *   out = (act(x·gateᵀ·s_g) * (x·upᵀ·s_u)) · downᵀ · s_d
 * x [T][D] bf16; out [T][D] in out_dtype (bf16 normally; f32 gives the
 * unrounded partial sum a tensor-parallel all-reduce wants).                */
size_t kw8_dense_ffn_workspace_size(int64_t T, int64_t D, int64_t H);
int kw8_dense_ffn(const void* x, int64_t T, int64_t D, int64_t H,
                  kw8_weight gate, kw8_weight up, kw8_weight down, int32_t act,
                  int32_t out_dtype, void* out, void* workspace,
                  size_t workspace_bytes, kw8_stream_t stream);

/* ------------------------------------------------------- W8 linears -- */

/* One W8 linear layer: out[t][n] = (Σ_k x[t][k] * q[n][k]) * s[n].
 * The attention projections of kappa (project_q / project_kv /
 * project_attn_out, kappa/qwen3/linear.py:11-25 and kappa/gemma3/linear.py:
 * 9-23) and the LM head (logits_from_hidden / _tied / _last_positions,
 * kappa/qwen3/transformer.py:55-75) are this product with kappa's weight
 * viewed K-major: w [N][K] int8 (N = heads*head_dim for Q/K/V, N = model dim
 * for O with K = heads*head_dim, N = vocab for the head).
 *   x    : bf16 rows of K features; row r of the product is x row
 *          rows[r] when `rows` (device int32 [T]) is given, else x row r
 *          (logits_from_hidden_last_positions gathers its rows this way).
 *   out  : [T][N] in out_dtype (kappa's einsum output is bf16).
 *   workspace >= kw8_linear_workspace_size(T, K, N) bytes.                  */
size_t kw8_linear_workspace_size(int64_t T, int64_t K, int64_t N);
int kw8_linear(const void* x, const int32_t* rows, int64_t T, int64_t K, int64_t N,
               kw8_weight w, int32_t out_dtype, void* out, void* workspace,
               size_t workspace_bytes, kw8_stream_t stream);

/* gather_embed_tokens (kappa/qwen3/quant.py:51-57) for a W8 table:
 * out[i][d] = dt(q[v][d]) * dt(s) with v = tokens[i], rounded once to
 * out_dtype, s the table's scale (per tensor, or per row v).  Ids follow a
 * JAX gather: a negative id counts from the end (v + V), then the id is
 * clamped into [0, V).  table.q is [V][D] int8; out [n][D].               */
int kw8_embed_gather(const int32_t* tokens, int64_t n, kw8_weight table, int64_t V,
                     int64_t D, int32_t out_dtype, void* out, kw8_stream_t stream);

/* ------------------------------------------------ norms + FFN sub-block -- */

/* rms_norm: out = bf16((f32(x) * rsqrt(mean(f32(x)^2) + eps)) * g),
 * g from kw8_norm_kind; x, out [T][D] bf16 (D % 8 == 0, D <= 16384);
 * scale [D] in scale_dtype.                                                 */
int kw8_rms_norm(const void* x, int64_t T, int64_t D, const void* scale, int32_t scale_dtype,
                 int32_t kind, float eps, void* out, kw8_stream_t stream);

/* The norms around a decoder block's FFN.  pre_scale [D] (required) is the
 * pre-FFN RMSNorm; post_scale [D] (or NULL: none, as in Qwen3) the post-FFN
 * RMSNorm; both in scale_dtype, of one kind.                                */
typedef struct kw8_block_norms {
  const void* pre_scale;
  const void* post_scale;
  int32_t scale_dtype;
  int32_t kind;
  float eps;
} kw8_block_norms;

/* The FFN sub-block of a dense decoder block, in one call:
 *   out = h + post_norm(FFN(pre_norm(h)))
 * with FFN = kw8_dense_ffn (act GELU_TANH: Gemma3, kappa/gemma3/block.py:
 * 73-82; act SILU and no post norm: Qwen3, kappa/qwen3/block.py:68-81).
 * Rounding as in kappa: the normed input, the FFN output, the post-normed
 * output and the sum are each bf16.  The down projection writes fp32
 * partial sums and one pass per row adds them, rounds, applies the post
 * norm and adds the residual.  h, out [T][D] bf16 (out may not alias h).  */
size_t kw8_dense_block_workspace_size(int64_t T, int64_t D, int64_t H);
int kw8_dense_block(const void* h, int64_t T, int64_t D, int64_t H, kw8_weight gate,
                    kw8_weight up, kw8_weight down, int32_t act, const kw8_block_norms* norms,
                    void* out, void* workspace, size_t workspace_bytes, kw8_stream_t stream);

/* ------------------------------------------------------------------ MoE -- */

/* Router of moe_swiglu_ffn: _route (kappa/qwen3/ffn_moe.py:38-56).
 *   logits[t][e] = Σ_d f32(x[t][d]) * f32(dequant(router))[d][e]   (fp32)
 *   top-k with ties to the lower expert index (jax.lax.top_k),
 *   w = bf16(softmax(top-k logits)).
 * router: [E][D] int8 (K-major view of kappa's [D, E]).
 * logits_out [T][E] f32 (may be workspace), idx_out [T][k] int32,
 * w_out [T][k] bf16.                                                         */
int kw8_moe_route(const void* x, int64_t T, int64_t D, int64_t E, int32_t k,
                  kw8_weight router, float* logits_out, int32_t* idx_out,
                  void* w_out, kw8_stream_t stream);

/* The top-k + softmax half of _route alone, on caller-provided logits.     */
int kw8_moe_topk(const float* logits, int64_t T, int64_t E, int32_t k,
                 int32_t* idx_out, void* w_out, kw8_stream_t stream);

/* Permutation of _moe_ragged (kappa/qwen3/ffn_moe.py:189-200): the stable
 * argsort of the flattened expert ids and bincount, plus the fixed-capacity
 * slot rule of _moe_fixed_capacity (ffn_moe.py:130-141).
 *   idx [T*k] int32 expert ids (row major [T][k]).
 *   capacity: rows kept per expert (slot < capacity); <0 means dropless.
 *   sorted_token [T*k]: token of each sorted row (only the first
 *       Σ group_sizes rows are written);
 *   inv_pos [T*k]: sorted row of flat entry i, or -1 if it was dropped;
 *   group_sizes [E] (rows kept), group_offsets [E+1] (exclusive prefix).    */
int kw8_moe_permute(const int32_t* idx, int64_t T, int32_t k, int64_t E,
                    int64_t capacity, int32_t* sorted_token, int32_t* inv_pos,
                    int32_t* group_sizes, int32_t* group_offsets,
                    kw8_stream_t stream);

/* kw8_moe_permute with scratch (same outputs): the sort runs over up to 148
 * blocks instead of one; workspace >= kw8_moe_permute_workspace_size(E)
 * bytes.  No counterpart in kappa beyond the function above.               */
size_t kw8_moe_permute_workspace_size(int64_t E);
int kw8_moe_permute_ws(const int32_t* idx, int64_t T, int32_t k, int64_t E,
                       int64_t capacity, int32_t* sorted_token, int32_t* inv_pos,
                       int32_t* group_sizes, int32_t* group_offsets,
                       void* workspace, size_t workspace_bytes, kw8_stream_t stream);

/* Expert FFN over permuted rows: the three ragged_dot calls and the SwiGLU
 * of _moe_ragged (kappa/qwen3/ffn_moe.py:202-210), run as grouped W8A16
 * GEMMs.  xs [rows][D] bf16 sorted by expert; group_offsets [E+1] on device;
 * gate/up [E][I][D], down [E][D][I] int8; ys [rows][D] bf16 where
 * rows = capacity of the buffers (T*k).                                     */
size_t kw8_moe_expert_ffn_workspace_size(int64_t rows, int64_t D, int64_t I,
                                         int64_t E);
int kw8_moe_expert_ffn(const void* xs, int64_t rows, int64_t D, int64_t I,
                       int64_t E, const int32_t* group_offsets,
                       kw8_weight gate, kw8_weight up, kw8_weight down,
                       void* ys, void* workspace, size_t workspace_bytes,
                       kw8_stream_t stream);

/* Combine / unpermute (kappa/qwen3/ffn_moe.py:212-215):
 *   out[t] = bf16( Σ_j f32(w[t][j]) * f32(ys[inv_pos[t*k+j]]) ), entries
 *   with inv_pos < 0 skipped.  fp32 sum in j order (kappa uses a bf16
 *   scatter-add whose order XLA chooses).                                   */
int kw8_moe_combine(const void* ys, const int32_t* inv_pos, const void* w,
                    int64_t T, int32_t k, int64_t D, void* out,
                    kw8_stream_t stream);

/* Whole MoE layer: moe_swiglu_ffn (kappa/qwen3/ffn_moe.py:226-299) for the
 * dropless implementations (ragged_jax, ragged_tokamax, gather_einsum —
 * mathematically the same function) and, with capacity >= 0, the
 * fixed_capacity one.  x [T][D] bf16 -> out [T][D] bf16.                    */
size_t kw8_moe_ffn_workspace_size(int64_t T, int64_t D, int64_t I, int64_t E,
                                  int32_t k);
int kw8_moe_ffn(const void* x, int64_t T, int64_t D, int64_t I, int64_t E,
                int32_t k, int64_t capacity, kw8_weight router,
                kw8_weight gate, kw8_weight up, kw8_weight down, void* out,
                void* workspace, size_t workspace_bytes, kw8_stream_t stream);

/* The FFN sub-block of a Qwen3 MoE decoder block (kappa/qwen3/block.py:
 * 68-81) in one call: out = h + post_norm(moe_swiglu_ffn(pre_norm(h))),
 * with the MoE layer of kw8_moe_ffn; the fp32 combine buffer goes through
 * one pass per row that rounds it, applies the post norm (if any) and adds
 * the residual.  h, out [T][D] bf16 (out may not alias h).                  */
size_t kw8_moe_block_workspace_size(int64_t T, int64_t D, int64_t I, int64_t E, int32_t k);
int kw8_moe_block(const void* h, int64_t T, int64_t D, int64_t I, int64_t E, int32_t k,
                  int64_t capacity, kw8_weight router, kw8_weight gate, kw8_weight up,
                  kw8_weight down, const kw8_block_norms* norms, void* out, void* workspace,
                  size_t workspace_bytes, kw8_stream_t stream);

/* ---------------------------------------------------- no-allocation -- */

/* kw8_moe_ffn with no workspace argument.  No counterpart in kappa (kappa
 * leaves memory to XLA); it exists for callers that cannot allocate device
 * memory where they call this library: e.g. a custom-call handler that is
 * given only its input and output buffers and no scratch allocator, or a
 * program whose device memory belongs to another allocator it cannot reach
 * from the call site.
 * The scratch is a fixed 16 MiB array inside the library; every GPU that
 * loads the library holds it until the process exits.  Shapes whose
 * kw8_moe_ffn_workspace_size() exceeds 16 MiB are rejected with
 * KW8_ERR_WORKSPACE (at the Qwen3-30B-A3B layer shape, D=2048, I=768,
 * E=128, k=8, that is above about 300 tokens).  The first call on each
 * device (and again after the device's context changed, e.g. after a
 * cudaDeviceReset) looks up the array's device address
 * (cudaGetSymbolAddress) and caches it; make that first call before any
 * stream capture.  Every call
 * on a device shares the one array, which keeps the last call's contents
 * (nothing in it needs to start at zero; the call clears what must), so
 * calls that overlap on the same GPU (other streams or threads) race and
 * corrupt each other's results.  Allocates nothing.                        */
int kw8_moe_ffn_noalloc(const void* x, int64_t T, int64_t D, int64_t I,
                        int64_t E, int32_t k, int64_t capacity,
                        kw8_weight router, kw8_weight gate, kw8_weight up,
                        kw8_weight down, void* out, kw8_stream_t stream);

/* ------------------------------------------------------ expert parallel -- */

/* Expert-parallel MoE row movement (no counterpart in kappa, which never
 * shards experts).  Rank r of `world` owns experts [r*E/world,
 * (r+1)*E/world).  counts [world][E] int32 (device): every rank's kept rows
 * per expert (an all-gather of group_sizes).  Every placement follows from
 * counts: rank r's receive buffer is expert-major, source-major within an
 * expert; a source's return buffer is in its permutation's (expert) order.
 * Rows move with plain peer-to-peer stores over NVLink into buffers mapped
 * with CUDA IPC; peer_recv / peer_out are device arrays of `world` mapped
 * addresses.  The caller orders the phases across ranks (a collective
 * between dispatch and the expert FFN, and between return and combine).
 *
 * kw8_ipc_*: device buffers shareable between the ranks' processes
 * (cudaMalloc + cudaIpcGetMemHandle, zero-filled before returning; handles
 * of kw8_ipc_handle_size() bytes are exchanged by the caller).             */
size_t kw8_ipc_handle_size(void);
int kw8_ipc_alloc(size_t bytes, void** ptr_out, void* handle_out);
int kw8_ipc_free(void* ptr);
int kw8_ipc_open(const void* handle, void** ptr_out);
int kw8_ipc_close(void* ptr);

/* Row p of this rank's sorted order (sorted_token / group_offsets from the
 * permutation, p < group_offsets[E] <= max_rows) -> x[sorted_token[p]]
 * written into its expert owner's receive buffer.  x [T][D] bf16.          */
int kw8_ep_dispatch(const void* x, int64_t max_rows, int64_t D,
                    const int32_t* sorted_token, const int32_t* group_offsets,
                    const int32_t* counts, int32_t world, int32_t rank,
                    int64_t E, const uint64_t* peer_recv, kw8_stream_t stream);

/* Rows of this rank's receive layout (expert outputs ys [rows][D] bf16,
 * rows <= max_rows) -> each written back to its source's return buffer at
 * the row's position in the source's sorted order.                        */
int kw8_ep_return(const void* ys, int64_t max_rows, int64_t D,
                  const int32_t* counts, int32_t world, int32_t rank, int64_t E,
                  const uint64_t* peer_out, kw8_stream_t stream);

/* Group offsets [E/world + 1] of this rank's receive layout (for
 * kw8_moe_expert_ffn on the received rows).                                */
int kw8_ep_local_offsets(const int32_t* counts, int32_t world, int32_t rank,
                         int64_t E, int32_t* local_offsets, kw8_stream_t stream);

/* An expert-parallel group as one rank sees it.  Every rank owns four
 * buffers, allocated with kw8_ipc_alloc and mapped by the others with
 * kw8_ipc_open; the device arrays hold each rank's mapping of them (this
 * rank's own buffer at [rank]):
 *   recv   : world * max_tokens * k rows of D bf16 (rows sent to this rank);
 *   out    : max_tokens * k rows of D bf16 (this rank's rows coming back);
 *   counts : int32 [2][world][E] (per-expert row counts of every rank, two
 *            copies alternating by call);
 *   flags  : uint32 [3][world] + 3 words, zero before the first call on any
 *            rank.
 * own_* are this rank's buffers again, as host-side values.
 *
 * With rows != NULL, kw8_moe_ffn_ep sends every token once per rank that
 * owns one of its experts instead of once per routed expert, and returns
 * one partial sum per token and rank; it then uses, instead of recv / out:
 *   rows : world * max_tokens rows of D bf16 (tokens sent to this rank);
 *   meta : world * max_tokens * k int32 row indices, then as many fp32
 *          routing weights (one record per routed pair);
 *   ret  : [world][max_tokens] rows of D partial sums coming back, in
 *          ret_format: KW8_RET_F32 (4*D bytes a row; the source rounds each
 *          output once, as one GPU does), KW8_RET_F16_SCALED (2*D bytes a
 *          row of fp16 values divided by a per-row power of two, then
 *          [world][max_tokens] fp32 scales after the rows: relative error
 *          per partial up to 2^-11) or KW8_RET_BF16 (2*D bytes, up to 2^-9);
 * and counts is int32 [2][world][E + world].                               */
/* Storage of the partial sums an expert-parallel step returns.            */
typedef enum kw8_ret_format {
  KW8_RET_BF16 = 0,
  KW8_RET_F32 = 1,
  KW8_RET_F16_SCALED = 2,
} kw8_ret_format;

typedef struct kw8_ep_peers {
  int32_t world;
  int32_t rank;
  int64_t max_tokens;
  const uint64_t* recv;
  const uint64_t* out;
  const uint64_t* counts;
  const uint64_t* flags;
  void* own_recv;
  void* own_out;
  int32_t* own_counts;
  uint32_t* own_flags;
  const uint64_t* rows;
  const uint64_t* meta;
  const uint64_t* ret;
  void* own_rows;
  void* own_meta;
  void* own_ret;
  int32_t ret_format; /* kw8_ret_format of the partial sums in ret        */
  /* Exchange buffer of the one-shot sums (kw8_moe_ffn_ep_decode,
   * kw8_dense_ffn_tp): fp32 [2][world][red_rows][D] in every rank.         */
  const uint64_t* red;
  float* own_red;
  int64_t red_rows;
} kw8_ep_peers;

/* The expert-parallel MoE layer over this rank's T <= max_tokens tokens in
 * one call, with no host synchronisation and no collective library: route,
 * permute, exchange the per-expert counts with every peer, write each
 * routed row into its expert owner's receive buffer, wait for every peer's
 * rows, run the local experts' FFN, write each output row back to its
 * source, wait for every peer, combine.  The phases are ordered by flag
 * words stored into the peers' memory (release/acquire at system scope)
 * and tagged with `epoch`, which must grow by one per call on every rank
 * of the group (start at 1).  gate/up/down hold this rank's E/world
 * experts.  Every wait is bounded (2 s): a peer that never arrives leaves
 * KW8_ERR_DEVICE_TIMEOUT in the device status (kw8_device_status) and an
 * unspecified `out`, but no hung kernel.  After a timeout the group is out
 * of step (a late peer may still store rows and counts into this rank's
 * buffers during its next call), so every rank must drop the group's
 * buffers or zero them again (after a host barrier) before calling again. */
size_t kw8_moe_ffn_ep_workspace_size(int64_t max_tokens, int64_t D, int64_t I, int64_t E,
                                     int32_t k, int32_t world);
int kw8_moe_ffn_ep(const void* x, int64_t T, int64_t D, int64_t I, int64_t E, int32_t k,
                   int64_t capacity, kw8_weight router, kw8_weight gate_local,
                   kw8_weight up_local, kw8_weight down_local, void* out,
                   const kw8_ep_peers* peers, uint32_t epoch, void* workspace,
                   size_t workspace_bytes, kw8_stream_t stream);

/* The expert-parallel MoE layer for a batch that every rank holds (decode,
 * kappa's moe_swiglu_ffn at small B*T), in one call: every rank routes all
 * T <= red_rows tokens (the same fp32 logits and top-k everywhere), runs
 * its own E/world experts' rows with the fused weighted combine into an
 * fp32 partial [T][D], stores that partial into every rank's exchange
 * buffer (peers->red, slot [epoch & 1][rank]), passes flag phase 1 of
 * `epoch`, and sums the world partials in rank order into out (bf16; every
 * rank gets the same bits).  Needs peers->red and peers->flags only
 * (epoch 0: the device-side call count of kw8_dense_ffn_tp).  No
 * counterpart in kappa, which replicates every expert.                     */
size_t kw8_moe_ffn_ep_decode_workspace_size(int64_t T, int64_t D, int64_t I, int64_t E, int32_t k);
int kw8_moe_ffn_ep_decode(const void* x, int64_t T, int64_t D, int64_t I, int64_t E, int32_t k,
                          int64_t capacity, kw8_weight router, kw8_weight gate_local,
                          kw8_weight up_local, kw8_weight down_local, void* out,
                          const kw8_ep_peers* peers, uint32_t epoch, void* workspace,
                          size_t workspace_bytes, kw8_stream_t stream);

/* Tensor-parallel dense FFN (the column/row split of kappa/qwen3/sharding.py:
 * 127-132, which kappa leaves to GSPMD) in one call: this rank's gate/up
 * shards ([H_local][D] each) and down shard ([D][H_local]) give an fp32
 * partial of the layer output; the partials are summed over the group like
 * kw8_moe_ffn_ep_decode's (peers->red, phase 1 of `epoch`) into out (bf16,
 * the same bits on every rank).  x [T][D] bf16 (the same on every rank),
 * T <= red_rows.
 * epoch: as for kw8_moe_ffn_ep, or 0: the group keeps the call count in
 * device memory (word 3 * world of each rank's flags), so a sequence of
 * calls captured in a CUDA graph takes a new tag at every replay.  Every
 * call of a group uses one of the two forms.  The sum runs as one
 * cooperative launch whose CTAs count themselves in flags words
 * 3 * world + 1 and + 2: the flags of a group that makes these calls hold
 * 3 * world + 3 words, zero before the first call.                         */
size_t kw8_dense_ffn_tp_workspace_size(int64_t T, int64_t D, int64_t H_local);
int kw8_dense_ffn_tp(const void* x, int64_t T, int64_t D, int64_t H_local, kw8_weight gate,
                     kw8_weight up, kw8_weight down, int32_t act, void* out,
                     const kw8_ep_peers* peers, uint32_t epoch, void* workspace,
                     size_t workspace_bytes, kw8_stream_t stream);

/* Milliseconds of the phases of the last timed kw8_moe_ffn_ep call on the
 * current device (option 4 set; deduplicated step), synchronising on it:
 * [0] route + permute, [1] slots + counts exchange (phase 0), [2] rows and
 * pair records to their owners, [3] wait for every peer's rows (phase 1),
 * [4] local offsets + gather of the received pairs, [5] expert FFN with the
 * fused combine, [6] partial sums back to their sources, [7] wait for every
 * peer's sums (phase 2), [8] final sum.  n <= 9 values are written.  No
 * counterpart in kappa.                                                    */
int kw8_ep_phase_times(float* ms_out, int32_t n);

/* Phase `phase` (0..2) of the group barrier: with `signal` this rank first
 * marks the phase done at every peer; then it waits (bounded) until every
 * rank has marked it for `epoch`.                                           */
int kw8_ep_barrier(const kw8_ep_peers* peers, int32_t phase, uint32_t epoch, int32_t signal,
                   kw8_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* KAPPA_W8_H_ */
