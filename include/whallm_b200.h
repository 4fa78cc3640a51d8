/*
 * whallm_b200 -- C ABI of the B200 routed-expert MoE path and the quantized
 * KV-cache formats.
 *
 * Every entry point:
 *   - takes caller-owned device pointers, plain sizes and a CUDA stream
 *     (wm_stream_t is the same type as cudaStream_t; pass NULL for the
 *     legacy default stream);
 *   - is asynchronous and stream-ordered, allocates no memory and keeps no
 *     state between calls (the tensor-core path caches a per-device tensor-map
 *     encoder lookup behind a mutex).  Exceptions, stated at each: the
 *     peer-exchange buffers of wep_ipc_alloc, and the installed-model loader
 *     wld_load_expert_layer, which is synchronous and keeps pinned host
 *     staging between calls;
 *   - returns WM_OK (0) or a negative WM_ERR_* code; w_last_error() then
 *     describes the failure for the calling thread.  No C++ exception crosses
 *     this boundary.
 *
 * bf16 tensors are passed as uint16_t bit patterns (wm_bf16).  All matrices
 * are row-major and densely packed.
 *
 * The reference (baha2046/Whallm) reaches the same operations through MLX
 * library calls; each declaration names the reference call site it replaces.
 * Paths are relative to the reference repository.
 */
#ifndef WHALLM_B200_H
#define WHALLM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define WM_API __attribute__((visibility("default")))
#else
#define WM_API
#endif

typedef struct CUstream_st *wm_stream_t;
typedef uint16_t wm_bf16;

#define WM_OK 0
#define WM_ERR_INVALID (-1)      /* bad argument, shape or alignment      */
#define WM_ERR_UNSUPPORTED (-2)  /* valid but not implemented shape       */
#define WM_ERR_CUDA (-3)         /* CUDA runtime error                    */
#define WM_ERR_WORKSPACE (-4)    /* workspace too small                   */

/* Output element types for dequantize calls. */
#define WM_OUT_F32 0
#define WM_OUT_BF16 1

/* Router score functions (deepseek_v41/moe.py:60-65, qwen4_exp.py:693). */
#define WM_SCORE_SOFTMAX 0
#define WM_SCORE_SIGMOID 1
#define WM_SCORE_SQRTSOFTPLUS 2
#define WM_SCORE_NONE 3
/* The Qwen gate in the reference's dtypes (qwen4_exp.py:683, 693-699): logits
 * rounded to bf16 (a bf16 nn.Linear), softmax(precise=True) in float32 rounded
 * to bf16, top-k on the bf16 probabilities, renormalised as bf16(p / bf16(sum)),
 * shared-expert gate bf16(sigmoid(bf16(logit))). */
#define WM_SCORE_SOFTMAX_BF16 4

/* Order of the fused gate/up projection rows. */
#define WM_UP_GATE 0 /* DeepSeek w13 = [w3(up); w1(gate)]  (expert_layout.py:43-60, model.py:417) */
#define WM_GATE_UP 1 /* Qwen gate_up = [gate; up]          (qwen4_exp.py:610, Qwen.swift:440)   */

/* KV-cache row formats. */
#define WKV_FP8_F32_B64 0   /* e4m3, one fp32 scale = amax/448 per 64 values                 */
#define WKV_FP8_UE8M0_B32 1 /* PackedRows 'fp8_ue8m0'  (deepseek_v41/packed_cache.py:24-59)   */
#define WKV_FP4_E4M3_B16 2  /* PackedRows 'fp4_e4m3'                                          */
#define WKV_FP4_UE8M0_B32 3 /* PackedRows 'fp4_ue8m0'                                         */
#define WKV_MXFP8_B32 4     /* mx.quantize(mode="mxfp8") chunks (fp8_cache.py:112)             */
#define WKV_MXFP4_B32 5     /* mx.quantize(mode="mxfp4") index copy (fp8_cache.py:116)         */

/* Message for the last failing call on this thread ("" if none). */
WM_API const char *w_last_error(void);
/* ABI version of this library. */
WM_API int w_abi_version(void);

/* ---------------------------------------------------------------- MXFP4 --- */

/* Quantize bf16 [rows, cols] (cols % 32 == 0) to MXFP4: packed e2m1 bytes
 * [rows, cols/2] (low nibble = even column) and E8M0 scales [rows, cols/32].
 * Replaces MXFP4.quantizeBF16 (Sources/DeepSeekRepack/MXFP4.swift:4-40); the
 * bytes are what mx.quantize(mode="mxfp4") stores (MXFP4.swift KATs,
 * Tests/DeepSeekRepackTests/DeepSeekRepackTests.swift:336-375). */
WM_API int wmxfp4_quantize(const wm_bf16 *src, int64_t rows, int64_t cols, uint8_t *packed,
                    uint8_t *scales, wm_stream_t stream);

/* Dequantize MXFP4 [rows, cols] to f32 or bf16 (out_dtype WM_OUT_*), bit-exact:
 * e2m1[code] * 2^(scale-127), code 8 -> +0.0.
 * Replaces dequant_fp4 (runtime/deepseek_v4_ssd/deepseek_v41/dequant.py:63-66)
 * and mx.dequantize(mode="mxfp4"). */
WM_API int wmxfp4_dequantize(const uint8_t *packed, const uint8_t *scales, int64_t rows, int64_t cols,
                      int out_dtype, void *out, wm_stream_t stream);

/* Exact two-term e4m3 form of bf16 rows, the token operand of the
 * block-scaled expert kernels: for each 32-value block, scale byte
 * s = clamp(exponent(block max) - 7, -122) + 127 (E8M0), hi = e4m3(x / 2^(s-127))
 * and lo = e4m3((x / 2^(s-127) - hi) * 2^5), both round-to-nearest-even, so
 * x = 2^(s-127) * (hi + 2^-5 * lo) exactly for every element within 2^-14 of
 * its block maximum.  hi, lo [rows, cols] u8, scales [rows, cols/32] u8.
 * No reference counterpart (an internal operand format); exported so the
 * decomposition can be checked bit for bit. */
WM_API int wmx_split_e4m3(const wm_bf16 *x, int rows, int cols, uint8_t *hi, uint8_t *lo, uint8_t *scales,
                   wm_stream_t stream);

/* Scores of queries against a quantized KV cache on block-scaled tensor cores:
 * scores[b, q, l] = bf16(query[b, q, :] . dequant(K)[b, l, :]) for a cache
 * stored as fmt = WKV_MXFP8_B32 (payload [B*L, D] e4m3, scales [B*L, D/32]
 * E8M0) or WKV_MXFP4_B32 (payload [B*L, D/2] e2m1, same scales).  query bf16
 * [B, Lq, D], scores bf16 [B, Lq, L]; D % 256 == 0.  Replaces
 * MXFP8PoolingCache.quantized_matmul / index_matmul over the completed chunks
 * (runtime/deepseek_v4_ssd/fp8_cache.py:119-159: mx.quantized_matmul,
 * transpose=True, group 32, mode mxfp8 / mxfp4).  Workspace:
 * wkv_scores_workspace_size(B, Lq, D, L); it includes room for f32 partial
 * sums when a decode-size launch (Lq <= 32) splits K to fill the GPU. */
WM_API size_t wkv_scores_workspace_size(int B, int Lq, int D, int L);
WM_API int wkv_mx_scores(const wm_bf16 *query, int B, int Lq, int D, const uint8_t *payload, const uint8_t *scales,
                  int L, int fmt, wm_bf16 *scores, void *workspace, size_t ws_bytes, wm_stream_t stream);

/* Dense block-scaled linear y [T, N] bf16 = x [T, K] bf16 @ dequant(w)^T for
 * w stored as fmt = WKV_MXFP8_B32 (u8 e4m3 [N, K]) or WKV_MXFP4_B32 (u8 e2m1
 * [N, K/2]) with E8M0 scales [N, K/32]; K % 256 == 0.  Replaces the MXFP8
 * QuantizedLinear layers nn.quantize(mode="mxfp8") installs over native FP8
 * weights (runtime/deepseek_v4_ssd/deepseek_v41_ssd.py:232-261, 353-360:
 * mx.quantized_matmul, transpose=True, group 32).  Workspace:
 * wmx_linear_workspace_size(T, K, N). */
WM_API size_t wmx_linear_workspace_size(int T, int K, int N);
WM_API int wmx_linear(const wm_bf16 *x, int T, int K, const uint8_t *w, const uint8_t *scales, int N, int fmt,
               wm_bf16 *y, void *workspace, size_t ws_bytes, wm_stream_t stream);

/* ------------------------------------ expert-parallel peer exchange ------ */

/* No reference counterpart (the reference is single-device).  The decode form
 * of the expert-parallel layer exchanges a few rows per rank per call over
 * NVLink without a collective library: buffers are shared with CUDA IPC,
 * rows are written straight into every rank's buffer and a per-rank flag is
 * raised there afterwards.  Epoch counters live in device memory (the calls
 * replay from CUDA graphs); all ranks make the same sequence of calls. */

/* cudaMalloc'd, zeroed buffer and its 64-byte IPC handle. */
WM_API int wep_ipc_alloc(size_t bytes, void **ptr, unsigned char *handle);
/* Map a peer's buffer from its handle / unmap / free. */
WM_API int wep_ipc_open(const unsigned char *handle, void **ptr);
WM_API int wep_ipc_close(void *ptr);
WM_API int wep_ipc_free(void *ptr);

/* For each of n_regions (<= 4) regions: rows x row_bytes from srcs[r]
 * (+ q * src_peer_stride[r] for peer q; src_peer_stride NULL: 0) to byte
 * dst_offsets[r] + rank * rows * row_bytes[r] of peer_dst[q], for every peer
 * q < world (<= 8, this rank included; row bytes, offsets and sources
 * 4-byte aligned, copied 16 bytes at a time where everything is 16-aligned);
 * then *epoch += 1 and
 * peer_flags[q][rank] = *epoch on every peer (release, system scope).
 * counter: a device int32 that starts at 0 and is left at 0. */
WM_API int wep_put_rows(int n_regions, const void *const *srcs, const size_t *row_bytes,
                 const size_t *src_peer_stride, const size_t *dst_offsets, int rows, void *const *peer_dst,
                 int rank, int world, uint32_t *const *peer_flags, uint32_t *epoch, int32_t *counter,
                 wm_stream_t stream);
/* Block the stream until flags[q] >= *epoch for all q < world (acquire,
 * system scope); after 2 s, *err = 1 and the wait ends. */
WM_API int wep_wait(const uint32_t *flags, int world, const uint32_t *epoch, int32_t *err, wm_stream_t stream);
/* out [rows, H] bf16 = sum over q < world of part[q] [rows, H] f32, in q
 * order; zeros when err != NULL and *err != 0. */
WM_API int wep_sum_rows(const float *part, int world, int rows, int H, const int32_t *err, wm_bf16 *out,
                 wm_stream_t stream);

/* ------------------------------------------------------ affine 4-bit ------ */

/* MLX-style affine 4-bit quantize, group `group` (64 or 32) along cols:
 * packed uint32 [rows, cols/8] (element 0 in the low nibble), bf16 scales and
 * biases [rows, cols/group].  Replaces mx.quantize(bits=4, group_size=64)
 * (shapes: runtime/deepseek_v4_ssd/deepseek_v41/engram.py:207-221). */
WM_API int waffine4_quantize(const wm_bf16 *src, int64_t rows, int64_t cols, int group, uint32_t *packed,
                      wm_bf16 *scales, wm_bf16 *biases, wm_stream_t stream);

/* w = scale*q + bias (float32), to f32 or bf16.  Replaces mx.dequantize(bits=4). */
WM_API int waffine4_dequantize(const uint32_t *packed, const wm_bf16 *scales, const wm_bf16 *biases,
                        int64_t rows, int64_t cols, int group, int out_dtype, void *out,
                        wm_stream_t stream);

/* Qwen QSA affine-quantized KV cache: mlx-lm QuantizedKVCache with group 32
 * and `bits` 4 or 8 (runtime/deepseek_v4_ssd/qwen_quantized_cache.py:6-20).
 * One tensor's cache (keys or values) is packed uint32
 * [n_seq, capacity, D*bits/32] (element 0 in the lowest bits) with bf16
 * scales and biases [n_seq, capacity, D/32]; n_seq = batch * kv heads.
 * append: quantize keys (and values, if not NULL) bf16 [n_seq, L, D] into
 * cache rows [offset, offset + L) of each sequence -- the quantize half of
 * update_and_fetch (qwen_quantized_cache.py:16).  Both tensors in one launch;
 * at most 2^34 values (n_seq * L * D) per tensor and call. */
WM_API int wkv_affine_append(const wm_bf16 *keys, const wm_bf16 *values, int64_t n_seq, int64_t L, int D,
                             int bits, uint32_t *k_q, wm_bf16 *k_s, wm_bf16 *k_b, uint32_t *v_q, wm_bf16 *v_s,
                             wm_bf16 *v_b, int64_t capacity, int64_t offset, wm_stream_t stream);

/* fetch: dequantize cache rows [0, L) of each sequence to bf16 [n_seq, L, D],
 * w = float32(scale) * q + float32(bias) rounded once -- the dequantize half
 * of update_and_fetch (qwen_quantized_cache.py:19-20).  values_out may be NULL. */
WM_API int wkv_affine_fetch(const uint32_t *k_q, const wm_bf16 *k_s, const wm_bf16 *k_b, const uint32_t *v_q,
                            const wm_bf16 *v_s, const wm_bf16 *v_b, int64_t n_seq, int64_t L, int64_t capacity,
                            int D, int bits, wm_bf16 *keys_out, wm_bf16 *values_out, wm_stream_t stream);

/* ------------------------------------------------------------- KV cache --- */

/* Quantize bf16 rows [rows, D] into payload [rows, D*bits/8] and scales
 * [rows, D/block] (float32 for WKV_FP8_F32_B64, one byte otherwise).
 * Replaces PackedRows.write (deepseek_v41/packed_cache.py:24-45) and the
 * mx.quantize calls of MXFP8PoolingCache.update (fp8_cache.py:109-117). */
WM_API int wkv_quantize(const wm_bf16 *x, int64_t rows, int D, int fmt, uint8_t *payload, void *scales,
                 wm_stream_t stream);

/* The e4m3 KV row formats by block and scale format (the forms named for
 * BASELINE config 5 and packed_cache.py 'fp8_ue8m0'): block 64 with one fp32
 * scale = amax/448 (WKV_SCALE_F32; WKV_FP8_F32_B64), or block 32 with a ue8m0
 * scale byte (WKV_SCALE_UE8M0; WKV_FP8_UE8M0_B32).  Other pairs return
 * WM_ERR_UNSUPPORTED.  Same results as wkv_quantize / wkv_dequantize. */
#define WKV_SCALE_F32 0
#define WKV_SCALE_UE8M0 1
WM_API int wkv_fp8_quantize(const wm_bf16 *x, int rows, int D, int block, int scale_fmt, uint8_t *payload,
                            void *scales, wm_stream_t stream);
WM_API int wkv_fp8_dequantize(const uint8_t *payload, const void *scales, int rows, int D, int block,
                              int scale_fmt, wm_bf16 *out, wm_stream_t stream);

/* Dequantize [rows, D] to bf16.  Replaces PackedRows.__getitem__
 * (packed_cache.py:47-59) and mx.dequantize in MXFP8PoolingCache._fetch
 * (fp8_cache.py:231-240). */
WM_API int wkv_dequantize(const uint8_t *payload, const void *scales, int64_t rows, int D, int fmt,
                   wm_bf16 *out, wm_stream_t stream);

/* Gather rows row_idx[n] (clipped to [0, rows-1]) and dequantize to bf16
 * [n, D].  Replaces the take_rows + mx.dequantize of
 * MXFP8PoolingCache.gather (fp8_cache.py:161-190). */
WM_API int wkv_gather_dequantize(const uint8_t *payload, const void *scales, int64_t rows,
                          const int32_t *row_idx, int64_t n, int D, int fmt, wm_bf16 *out,
                          wm_stream_t stream);

/* --------------------------------------------------------------- router --- */

/* Gate logits, scores, top-k and weights for T tokens.
 *   logits[t,e] = x[t].wg[e] (float32, fixed order) + logit_bias[e] (if given)
 *   score       = score_fn(logits)           (softmax over E, sigmoid, sqrt(softplus), none,
 *                                             or WM_SCORE_SOFTMAX_BF16: the bf16 gate above)
 *   selection   = top-k of score + select_bias (bias picks, does not scale;
 *                 deepseek_v41/moe.py:67-70), ties to the lower expert id
 *                 (model.py:548-560); idx is in selection order
 *   weights     = score[idx] / (sum + norm_eps) if norm_eps >= 0, times route_scale
 *                 (deepseek_v41/moe.py:71-73: eps 1e-20, scale 1.5;
 *                  qwen4_exp.py:696-697: eps 0, scale 1)
 *   shared_w[t] = sigmoid(x[t].wg_shared) if wg_shared (qwen4_exp.py:699).
 * logits [T,E] float32 is caller-provided scratch and receives the biased logits.
 * Replaces Gate.__call__ (deepseek_v41/moe.py:58-75) and the routing half of
 * SparseMoE.__call__ (qwen4_exp.py:692-697).  H % 8 == 0, E <= 1024, k <= 32. */
WM_API int wmoe_router_topk(const wm_bf16 *x, const wm_bf16 *wg, const float *logit_bias,
                     const float *select_bias, const wm_bf16 *wg_shared, int T, int H, int E, int k,
                     int score_fn, float norm_eps, float route_scale, float *logits, int32_t *idx,
                     float *weights, float *shared_w, wm_stream_t stream);

/* The score / top-k / renormalisation half of wmoe_router_topk on caller
 * logits [T,E] (float32).  With WM_SCORE_NONE and norm_eps < 0 this is the
 * positional-tie top-k of _stable_topk_indices (model.py:548-560) in
 * selection order; it also serves gates whose logits come from elsewhere
 * (mlx-lm MoEGate, called at dspark.py:32). */
WM_API int wmoe_topk_scores(const float *logits, const float *select_bias, int T, int E, int k,
                            int score_fn, float norm_eps, float route_scale, int32_t *idx,
                            float *weights, wm_stream_t stream);

/* wmoe_router_topk without the logits scratch argument, for callers that
 * cannot call cudaMalloc where they route (serving loops that must stay free
 * of device allocations, hosts whose device memory belongs to another
 * allocator).  No counterpart in the reference: MLX allocates its own
 * temporaries.  The [T,E] logits live in a 1 MiB file-scope device array
 * (T*E <= 262144, else WM_ERR_INVALID), reserved on every GPU that loads the
 * library until exit and shared by all calls: calls that overlap on the GPU
 * race.  The array's address is looked up on the first call per device and
 * kept; make that first call before any stream capture.  The kept address
 * belongs to the device's context at that time: after cudaDeviceReset (a new
 * context) the address is stale, so do not use this entry point after a
 * reset.  Results equal wmoe_router_topk's. */
WM_API int wmoe_router_topk_static(const wm_bf16 *x, const wm_bf16 *wg, const float *logit_bias,
                                   const float *select_bias, const wm_bf16 *wg_shared, int T, int H,
                                   int E, int k, int score_fn, float norm_eps, float route_scale,
                                   int32_t *idx, float *weights, float *shared_w, wm_stream_t stream);

/* -------------------------------------------------------------- permute --- */

/* Stable sort of the T*k assignments by expert (mlx-lm _gather_sort, called at
 * model.py:404 and qwen4_exp.py:622): offsets [E+1], perm [T*k] (sorted slot
 * -> flat assignment t*k+j), inv [T*k] (flat -> sorted slot; _scatter_unsort).
 * The ids are checked on the device: if any is outside [0, E), offsets[E] is
 * set to -1 and perm/inv are left unwritten. */
WM_API int wmoe_permute(const int32_t *idx, int T, int k, int E, int32_t *offsets, int32_t *perm,
                 int32_t *inv, wm_stream_t stream);

/* ------------------------------------------------------ expert forward ---- */

/* Workspace bytes for wmoe_*_experts / wmoe_*_moe_forward. */
WM_API size_t wmoe_workspace_size(int T, int k, int H, int I, int E, int has_shared);

/* Routed experts, un-reduced: out[t, j, :] = FFN_{idx[t,j]}(x[t]) in bf16 [T,k,H].
 * Experts are stacked MXFP4: w13 [E, 2I, H/2] + s13 [E, 2I, H/32],
 * w2 [E, H, I/2] + s2 [E, H, I/32].  FFN = down(act(split(w13 x))) with
 * ClampedSwiGLU(limit) (limit 0: plain SwiGLU).
 * Replaces _StreamingSwitchGLU.__call__ / _gather_qmm (model.py:283-459) and
 * StreamingExperts.__call__ (qwen4_exp.py:613-678). */
WM_API int wmoe_mxfp4_experts(const wm_bf16 *x, const int32_t *idx, int T, int k, int H, int I, int E,
                       const uint8_t *w13, const uint8_t *s13, const uint8_t *w2, const uint8_t *s2,
                       int gate_up_order, float swiglu_limit, wm_bf16 *out, void *workspace,
                       size_t ws_bytes, wm_stream_t stream);

/* Routed experts + top-k weighted combine (+ shared expert): out [T,H] bf16 =
 *   sum_j weights[t,j] * FFN_{idx[t,j]}(x[t]) + shared_w[t] * FFN_{shared}(x[t])
 * in float32.  shared_expert < 0: none; shared_w NULL: weight 1.
 * Replaces _streaming_moe + _route_reduce (model.py:484-504), MoE.__call__
 * (deepseek_v41/moe.py:105-112) and SparseMoE.__call__ (qwen4_exp.py:692-704). */
WM_API int wmoe_mxfp4_moe_forward(const wm_bf16 *x, const int32_t *idx, const float *weights, int T, int k,
                           int H, int I, int E, const uint8_t *w13, const uint8_t *s13,
                           const uint8_t *w2, const uint8_t *s2, int gate_up_order,
                           float swiglu_limit, int shared_expert, const float *shared_w,
                           wm_bf16 *out, void *workspace, size_t ws_bytes, wm_stream_t stream);

/* One whole routed-expert layer: wmoe_router_topk followed by
 * wmoe_mxfp4_moe_forward on its outputs, in one call and on one stream, with
 * the same results bit for bit (logits, idx, weights, shared_w and out are
 * all written).
 *   router:  gate wg [n_routed, H], logit_bias, select_bias, wg_shared, k,
 *            score_fn, norm_eps, route_scale as wmoe_router_topk;
 *   experts: E = n_routed (+1 when shared_expert >= 0, which must then be
 *            n_routed: the shared expert is the last one), weighted by
 *            shared_w when wg_shared is given, else by 1.
 * Workspace: wmoe_workspace_size(T, k, H, I, E, shared_expert >= 0).  Replaces MoE.__call__
 * (deepseek_v41/moe.py:105-112) and SparseMoE.__call__ (qwen4_exp.py:680-704)
 * with their gates. */
WM_API int wmoe_mxfp4_moe_layer(const wm_bf16 *x, int T, int H, int I, const wm_bf16 *wg, const float *logit_bias,
                                const float *select_bias, const wm_bf16 *wg_shared, int n_routed, int k,
                                int score_fn, float norm_eps, float route_scale, const uint8_t *w13,
                                const uint8_t *s13, const uint8_t *w2, const uint8_t *s2, int gate_up_order,
                                float swiglu_limit, int shared_expert, float *logits, int32_t *idx, float *weights,
                                float *shared_w, wm_bf16 *out, void *workspace, size_t ws_bytes,
                                wm_stream_t stream);

/* One expert-parallel rank's share of wmoe_mxfp4_moe_forward, for decode
 * after an all-gather of every rank's tokens (T = all ranks' tokens):
 * out [T,H] float32 = sum over j with idx[t,j] in [route_base,
 * route_base + route_count) of weights[t,j] * FFN_{idx[t,j] - route_base}(x[t])
 * + (shared_lo <= t < shared_hi ? shared_w[t] * FFN_{shared}(x[t]) : 0).
 * The weight tensors hold E_local experts: the rank's route_count routed
 * experts, then (optionally) the shared expert at index shared_expert.  Ids in
 * [0, n_routed) owned by other ranks are skipped; ids outside [0, n_routed)
 * set the error path (zeros).  `placement` (NULL, or int32 [n_routed] holding
 * a permutation of [0, n_routed)) moves routed id e to position
 * placement[e]: the rank then owns the ids whose positions lie in
 * [route_base, route_base + route_count), local expert = position -
 * route_base -- a popularity-balanced assignment of experts to ranks with the
 * router's ids unchanged.  Summing `out` over the ranks (a reduce-scatter
 * over the token blocks) gives the layer output.  The reference has no
 * multi-device MoE (_streaming_moe raises on a sharding group,
 * model.py:485-486); this is the sharded form of the same layer.  Workspace:
 * wmoe_workspace_size(T, k, H, I, E_local, shared_expert >= 0). */
WM_API int wmoe_mxfp4_moe_forward_ep(const wm_bf16 *x, const int32_t *idx, const float *weights, int T, int k,
                              int H, int I, int E_local, int n_routed, int route_base, int route_count,
                              const int32_t *placement, const uint8_t *w13, const uint8_t *s13, const uint8_t *w2, const uint8_t *s2,
                              int gate_up_order, float swiglu_limit, int shared_expert, const float *shared_w,
                              int shared_lo, int shared_hi, float *out, void *workspace, size_t ws_bytes,
                              wm_stream_t stream);

/* Top-k weighted reduce of expert rows: out [T, H] bf16 =
 *   sum_j weights[t, j] * y[slots[t, j], :]  (+ add[t, :] if add != NULL)
 * accumulated in float32 in j order (fmaf), the addend last, rounded once.
 * y: [rows, H] bf16; slots [T, k] int32 (a slot outside [0, rows) is
 * skipped); add: float32 [T, H] (e.g. a gated shared expert) or NULL.
 * Replaces _route_reduce (runtime/deepseek_v4_ssd/model.py:502-504, with
 * slots t * k + j over the un-reduced switch_mlp rows) and the combine of an
 * expert-parallel layer whose rows came back through an all-to-all. */
WM_API int wmoe_route_reduce(const wm_bf16 *y, int64_t rows, const int32_t *slots, const float *weights, int T,
                             int k, int H, const float *add, wm_bf16 *out, wm_stream_t stream);

/* Affine 4-bit experts (group `group`): w13 uint32 [E, 2I, H/8] with bf16
 * sc13/bi13 [E, 2I, H/group]; w2 uint32 [E, H, I/8] with sc2/bi2 [E, H, I/group]. */
WM_API int wmoe_affine4_experts(const wm_bf16 *x, const int32_t *idx, int T, int k, int H, int I, int E,
                         const uint32_t *w13, const wm_bf16 *sc13, const wm_bf16 *bi13,
                         const uint32_t *w2, const wm_bf16 *sc2, const wm_bf16 *bi2, int group,
                         int gate_up_order, float swiglu_limit, wm_bf16 *out, void *workspace,
                         size_t ws_bytes, wm_stream_t stream);

WM_API int wmoe_affine4_moe_forward(const wm_bf16 *x, const int32_t *idx, const float *weights, int T,
                             int k, int H, int I, int E, const uint32_t *w13, const wm_bf16 *sc13,
                             const wm_bf16 *bi13, const uint32_t *w2, const wm_bf16 *sc2,
                             const wm_bf16 *bi2, int group, int gate_up_order, float swiglu_limit,
                             int shared_expert, const float *shared_w, wm_bf16 *out,
                             void *workspace, size_t ws_bytes, wm_stream_t stream);

/* Installed-model expert layer -> device tensors.  `path` is an installed
 * `experts/layer_XX.bin`: n_blobs expert blobs of blob_size bytes (the file
 * size must equal n_blobs * blob_size; manifest.py:170-175).  For every region
 * r and blob b, bytes [src_offsets[r], src_offsets[r] + lengths[r]) of blob b
 * are copied to device memory dst_bases[r] + b * dst_pitches[r].  This
 * replaces the per-blob slot copies of the expert cache (_SlotPool.store,
 * expert_cache.py:416-428, into the slot layout of expert_layout.py:8-80): a
 * caller that points w3 and w1 (or their scales) at the two halves of each
 * expert's rows in one [E, 2I, ...] tensor gets the fused w13 = [w3; w1].
 * The file is read in chunks of whole blobs (about chunk_bytes each), by up
 * to 8 threads, into two pinned buffers that the library keeps (and grows)
 * across calls until exit; concurrent calls are serialised.  Returns after
 * every copy on `stream` has completed. */
WM_API int wld_load_expert_layer(const char *path, size_t blob_size, int n_blobs, int n_regions,
                                 const size_t *src_offsets, const size_t *lengths, void *const *dst_bases,
                                 const size_t *dst_pitches, size_t chunk_bytes, wm_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* WHALLM_B200_H */
