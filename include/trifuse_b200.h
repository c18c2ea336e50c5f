/*
 * trifuse_b200.h - C ABI of the B200 (sm_100a) OLMoE sparse-MoE forward path.
 *
 * Drop-in boundary for the path that TriFuse's MLX model adapter runs:
 * the router, MLX-affine 4-bit gather_qmm, SwiGLU, the top-k combine and the
 * fp16 KV-cache attention with full-width Q/K RMSNorm and RoPE.  Each entry
 * point names the reference interface it replaces (paths relative to the
 * TriFuse project root; line numbers inside patches/executorch.patch are
 * lines of the patch file).
 *
 * Conventions
 *  - Every function returns a tf_status.  Nothing throws across the ABI; the
 *    text of the last failure on the calling thread is tf_last_error().
 *    (Replaces need()/std::runtime_error, MLXNativeGraniteMoEPrefill.h:520-522,
 *    and MLXBackend::execute's Error::Internal mapping,
 *    patches/executorch.patch:1486-1499.)
 *  - Tensor arguments are plain device pointers with explicit sizes, row-major
 *    and contiguous, unless a parameter says "host".  `stream` is a
 *    cudaStream_t passed as void* (NULL = the legacy default stream).
 *  - Shape and argument checks happen before any launch; a failed check
 *    launches nothing and changes no output.  Route counts (tokens * k) are
 *    limited to 2^31 - 1.
 *  - Index arrays that live on the device (expert ids, token and route
 *    indices, attention positions) are read only by the kernels and are not
 *    range-checked on the host: ids outside [0, experts), rows outside
 *    [0, x_rows) or positions outside [0, max_length) are undefined
 *    behaviour, as out-of-range indices are in MLX's gather_qmm.  Token ids
 *    of the embedding are the exception: a negative id reads row 0 (the
 *    reference's maximum(token, 0)), and an id past the table reads row 0
 *    and records device error 6 (tf_device_error).  Host-resident ids
 *    (session calls with TF_HOST_INPUTS) are checked before any launch, and
 *    the Python mirror (trifuse_b200.ops) checks device ids on the host.
 *  - Activation tensors ("act") are float16 or bfloat16 (tf_dtype).  Packed
 *    weights are uint32 words holding eight 4-bit codes, code j at bits 4j;
 *    scales and biases are float16, one per group of 64 inputs
 *    (overlays/executorch/backends/mlx/native_affine_ops.py:12-36).
 *  - Functions marked "workspace" take caller-owned device scratch of at least
 *    the size their *_workspace_size companion reports; they allocate nothing.
 */
#ifndef TRIFUSE_B200_H
#define TRIFUSE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TF_ABI_VERSION 1

typedef enum tf_status {
  TF_OK = 0,
  TF_ERR_INVALID_ARGUMENT = 1,
  TF_ERR_SHAPE = 2,
  TF_ERR_OUT_OF_MEMORY = 3,
  TF_ERR_CUDA = 4,
  TF_ERR_NCCL = 5,
  TF_ERR_TIMEOUT = 6,
  TF_ERR_CANCELLED = 7,
  TF_ERR_UNSUPPORTED = 8,
  TF_ERR_STATE = 9,
  TF_ERR_CAPACITY = 10
} tf_status;

typedef enum tf_dtype {
  TF_DTYPE_F16 = 1,
  TF_DTYPE_BF16 = 2,
  TF_DTYPE_F32 = 3
} tf_dtype;

/* MLX affine-quantized weight, stacked over experts when experts > 0.
 * q: uint32 [E][out][in*bits/32]; scales, biases: f16 [E][out][in/group].
 * experts == 0 means a plain 2-D weight.  Only bits 4 / group 64 run here;
 * anything else is TF_ERR_UNSUPPORTED.
 * Mirrors the Q/S/B binding of MLXNativeGraniteMoEPrefill.h:220-262. */
typedef struct tf_affine_weight {
  const uint32_t* q;
  const void* scales;
  const void* biases;
  int32_t experts;
  int32_t out_features;
  int32_t in_features;
  int32_t group_size;
  int32_t bits;
} tf_affine_weight;

/* Router weight: dense act [experts][hidden] when `dense` is non-NULL,
 * otherwise the affine weight (the model's 4-bit mlp.gate,
 * tools/export/export_native_olmoe_target.py:74). */
typedef struct tf_router_weight {
  const void* dense;
  tf_affine_weight affine;
} tf_router_weight;

/* ------------------------------------------------------------------------ */
/* library                                                                    */

int tf_abi_version(void);
const char* tf_last_error(void);
const char* tf_status_name(int status);
/* TF_OK when `device` is an sm_100 GPU and this library's kernels load on it. */
int tf_device_check(int device);
/* Kernels this library has launched since it was loaded (all threads).
 * Diagnostic counter; no reference counterpart beyond the env-gated timing
 * lines of src/apple/TFETResidentSession.mm:48-83. */
uint64_t tf_launch_count(void);
/* Kernel path for the 4-bit QMMs: 0 = automatic (tensor cores when a weight
 * matrix serves enough tokens), 1 = CUDA-core GEMV only, 2 = tensor cores
 * whenever the shape allows.  Process-wide; for A/B checks and timing.
 * The reference's analogue is TRIFUSE_SORTED_QMM_BM (patches/mlx.patch:
 * 186-206) selecting its gather_qmm tile. */
int tf_set_qmm_path(int path);
/* First error code recorded by a device-side bounded wait since the last
 * clear (0 = none): a tensor-core tile whose pipeline stalled past its
 * limit returns early instead of hanging.  Synchronizes the device. */
int tf_device_error(int clear);

/* ------------------------------------------------------------------------ */
/* operators (graph-level surface)                                            */

/* y[r] = act((x*r) * w), r = 1/sqrt(mean(x^2) + eps); width % 256 == 0.
 * Replaces fast::rms_norm at MLXNativeGraniteMoEPrefill.h:434, 451-452, 486, 490. */
int tf_rms_norm(const void* x, int64_t rows, int32_t width, const void* weight_f16,
                float eps, int act, void* y, void* stream);

/* y[rows][out] = act(x[rows][in] . dequant(W)^T), fp32 accumulation.
 * Replaces mlx::native_affine_qmm (native_affine_ops.py:39-52) /
 * quantized_matmul (MLXNativeGraniteMoEPrefill.h:539-541). */
int tf_affine_qmm(const void* x, int64_t rows, const tf_affine_weight* w, int act,
                  void* y, void* stream);

/* Row n of y uses expert indices[n] and input row x_index[n] (or n / rows_per_x
 * when x_index is NULL, which is the broadcast form x[1,T,1,1,H] x idx[1,T,K]
 * with rows_per_x = K):  y[n] = act(x[row] . dequant(W[indices[n]])^T).
 * sorted_indices is the caller's promise that indices never decrease (as in
 * the reference it only selects a schedule, never the result).
 * Replaces mlx::native_affine_gather_qmm (native_affine_ops.py:55-74) /
 * gather_qmm (MLXNativeGraniteMoEPrefill.h:542-550). */
int tf_affine_gather_qmm(const void* x, int64_t x_rows, int32_t rows_per_x,
                         const int32_t* x_index, const int32_t* indices, int64_t n,
                         const tf_affine_weight* w, int sorted_indices, int act, void* y,
                         void* stream);

/* y[n] = dequant(table[ids[n]]) rounded to out_dtype (f16 in the reference).
 * Replaces mlx::native_affine_embedding (native_affine_ops.py:77-93) and the
 * selected-row dequantize of MLXNativeGraniteMoEPrefill.h:394-396. */
int tf_affine_embedding(const int64_t* ids, int64_t n, const tf_affine_weight* table,
                        int out_dtype, void* y, void* stream);

/* probs = act(softmax_fp32(logits)); experts <= 64.
 * Replaces mlx::native_olmoe_softmax (native_affine_ops.py:128-138). */
int tf_olmoe_softmax(const void* logits, int64_t rows, int32_t experts, int act,
                     void* probs, void* stream);

/* indices[r] = first k of the stable descending rank of probs[r] (NaN last,
 * ties to the lower expert id), int32.
 * Replaces mlx::native_olmoe_topk_indices (native_affine_ops.py:141-153). */
int tf_olmoe_topk_indices(const void* probs, int64_t rows, int32_t experts, int32_t k,
                          int act, int32_t* indices, void* stream);

/* out[r][j] = x[r][indices[r][j]].
 * Replaces mlx::native_take_along_last (native_affine_ops.py:115-125). */
int tf_take_along_last(const void* x, int64_t rows, int32_t width, const int32_t* indices,
                       int32_t k, int act, void* out, void* stream);

/* Top-k combine + residual: out[t] = act(residual[t] + act(sum_k act(y[inverse[t*k+j]]
 * * gates[t][j]))), the fp32 sum taken in k order from the k = 0 product.
 * y_sorted act [tokens*k][hidden] (rows in route-sort order), inverse int32
 * [tokens*k], gates act [tokens][k]; hidden % 8 == 0.
 * Replaces the combine of moe() (MLXNativeGraniteMoEPrefill.h:688-695). */
int tf_moe_combine(const void* y_sorted, const int32_t* inverse, const void* gates, const void* residual,
                   int64_t tokens, int32_t k, int32_t hidden, int act, void* out, void* stream);

/* Softmax + rank + take in one launch: (indices int32 [T][k] in rank order,
 * gates act [T][k]).  No top-k renormalisation.
 * Replaces olmoe_route (overlays/executorch/backends/mlx/runtime/
 * MLXOLMoERouter.h:86-120) and route() (MLXNativeGraniteMoEPrefill.h:591-602). */
int tf_olmoe_route(const void* logits, int64_t tokens, int32_t experts, int32_t k, int act,
                   int32_t* indices, void* gates, void* stream);

/* Router GEMV + route in one launch: logits = act(x . W_r^T) in a fixed fp32
 * order, then as tf_olmoe_route.  `logits` may be NULL.  hidden % 256 == 0.
 * Replaces linear(x, layer.router) + route() (MLXNativeGraniteMoEPrefill.h:631-632). */
int tf_olmoe_router(const void* x, int64_t tokens, int32_t hidden,
                    const tf_router_weight* router, int32_t experts, int32_t k, int act,
                    void* logits, int32_t* indices, void* gates, void* stream);

/* Stable grouping of the T*k routes by expert (workspace):
 * order = stable argsort(flat indices), inverse = its inverse permutation,
 * offsets[e] = first sorted slot of expert e (experts + 1 entries).
 * Replaces the sort of MLXNativeGraniteMoEPrefill.h:666-684. */
int tf_moe_route_sort_workspace_size(int64_t tokens, int32_t k, int32_t experts, size_t* bytes);
int tf_moe_route_sort(const int32_t* indices, int64_t tokens, int32_t k, int32_t experts,
                      int32_t* order, int32_t* inverse, int32_t* offsets, void* workspace,
                      size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* MoE block                                                                  */

typedef struct tf_moe_args {
  const void* x;         /* act [tokens][hidden]: post-attention-norm hidden   */
  const void* residual;  /* act [tokens][hidden]                               */
  void* out;             /* act [tokens][hidden] = residual + sum_k g_k E_k(x) */
  int64_t tokens;
  int32_t hidden;        /* % 256 == 0 */
  int32_t intermediate;  /* % 64 == 0  */
  int32_t experts;       /* <= 64      */
  int32_t top_k;         /* <= 32      */
  int32_t act;           /* tf_dtype   */
  tf_router_weight router;
  tf_affine_weight gate_proj; /* [experts][intermediate][hidden] */
  tf_affine_weight up_proj;   /* [experts][intermediate][hidden] */
  tf_affine_weight down_proj; /* [experts][hidden][intermediate] */
  void* logits;          /* optional act [tokens][experts] */
  int32_t* indices;      /* optional [tokens][top_k]       */
  void* gates;           /* optional act [tokens][top_k]   */
} tf_moe_args;

/* One sparse-MoE block (workspace): router, route, sort, gate/up gather_qmm
 * with fused SwiGLU, down gather_qmm, weighted combine + residual.
 * Replaces NativeGraniteMoEPrefill::moe (MLXNativeGraniteMoEPrefill.h:627-702)
 * = MoE.forward + residual (tools/export/export_native_olmoe_target.py:200-218, 227). */
int tf_moe_workspace_size(const tf_moe_args* args, size_t* bytes);
int tf_moe_forward(const tf_moe_args* args, void* workspace, size_t workspace_bytes,
                   void* stream);

/* The MoE block for callers that cannot allocate device memory while it runs
 * (a host framework's execute callback with a pre-planned memory arena, or a
 * serving loop where cudaMalloc/cudaFree would synchronize the device):
 * same computation and arguments as tf_moe_forward, but no workspace
 * argument and no allocation by this library.  Its scratch is one fixed
 * TF_MOE_NOALLOC_SCRATCH_BYTES buffer built into this library, held on every
 * GPU that loads it.  Calls with more than TF_MOE_NOALLOC_MAX_TOKENS tokens,
 * or whose scratch would exceed the buffer (it fits 64 tokens at
 * OLMoE-1B-7B geometry), return TF_ERR_CAPACITY.  Without the workspace this
 * entry runs every tensor-core tile on one block (no split schedule).
 * The first call on a device looks up the buffer's device address, so make
 * it before any stream capture; the address is kept for the process, so do
 * not use this entry across a reset of the device (cudaDeviceReset).  With
 * CUDA's lazy module loading (the default) the first call on a device, and
 * the first call of each batch shape, may still load kernel modules, which
 * allocates device memory and synchronizes inside the driver: callers that
 * must never see that make one warm-up call per device and shape, or run
 * with CUDA_MODULE_LOADING=EAGER.  All calls share the buffer: calls that
 * overlap on the GPU race and must be serialized.  No counterpart in the
 * reference. */
#define TF_MOE_NOALLOC_SCRATCH_BYTES ((size_t)6 << 20)
#define TF_MOE_NOALLOC_MAX_TOKENS 64
int tf_moe_forward_noalloc(const tf_moe_args* args, void* stream);

/* The expert hook's GPU callable (workspace): for parallel route vectors
 * (token_indices[n], expert_ids[n]) return out_sorted [n][hidden], the expert
 * outputs in expert-sorted order, and inverse [n] so that
 * out_sorted[inverse[i]] belongs to route i.  experts_sorted is the caller's
 * promise that expert_ids never decrease.  n == 0 is allowed.
 * Replaces NativeMoEExpertHook::GPUCallable (overlays/executorch/backends/mlx/
 * runtime/MLXMoEExpertHook.h:25-32; body MLXNativeGraniteMoEPrefill.h:635-658). */
int tf_moe_expert_workspace_size(int64_t n, int64_t x_rows, int32_t hidden, int32_t intermediate,
                                 int32_t experts, int act, size_t* bytes);
int tf_moe_expert_gpu(const void* x, int64_t x_rows, int32_t hidden, const int32_t* token_indices,
                      const int32_t* expert_ids, int64_t n, int experts_sorted,
                      int32_t intermediate, int32_t experts, const tf_affine_weight* gate_proj,
                      const tf_affine_weight* up_proj, const tf_affine_weight* down_proj, int act,
                      void* out_sorted, int32_t* inverse, void* workspace, size_t workspace_bytes,
                      void* stream);

/* The expert hook's computation with the outputs in the routes' own order:
 * out [n][hidden] row i belongs to route i (token_indices[i], expert_ids[i]).
 * Same workspace as tf_moe_expert_gpu.  For the expert-parallel layer,
 * whose received rows go back to their ranks in the order they came; no
 * counterpart in the reference (its hook returns expert-sorted rows and the
 * inverse permutation). */
int tf_moe_expert_gpu_ordered(const void* x, int64_t x_rows, int32_t hidden, const int32_t* token_indices,
                              const int32_t* expert_ids, int64_t n, int32_t intermediate, int32_t experts,
                              const tf_affine_weight* gate_proj, const tf_affine_weight* up_proj,
                              const tf_affine_weight* down_proj, int act, void* out, void* workspace,
                              size_t workspace_bytes, void* stream);

/* y[i] = x[index[i] / div] for i < n: act rows of `width` (% 8 == 0); x has
 * x_rows rows.  The routed-row gather x[order // k] of the MoE dispatch
 * (MLXNativeGraniteMoEPrefill.h:670-684), used by the expert-parallel layer
 * to fill its send buffer. */
int tf_gather_rows(const void* x, int64_t x_rows, int32_t width, const int32_t* index, int32_t div, int64_t n,
                   int act, void* y, void* stream);

/* ------------------------------------------------------------------------ */
/* attention                                                                  */

/* One decode step of attention for `batch` independent requests (workspace).
 * qkv: act [batch][3*heads*head_dim] = q | k | v projections of this token.
 * Full-width RMSNorm of q and k (q_norm/k_norm f16 [heads*head_dim]), RoPE
 * (half-split, theta) at positions[b], append k/v (as f16) at slot positions[b]
 * of the request's cache, then softmax(q K^T * scale) V over slots
 * [0, positions[b]] -> out act [batch][heads*head_dim].  positions is a
 * device array; max_length bounds positions[b] + 1 (pass capacity when
 * unknown).  Only head_dim 128 runs here.
 * Cache layout: k_cache/v_cache f16 [batch][heads][capacity][head_dim].
 * Replaces MLXNativeGraniteMoEPrefill.h:446-483 for T == 1 (q/k/v already
 * projected), including MLXSequenceCache::update_and_fetch
 * (patches/executorch.patch:3357-3405). */
int tf_attention_decode_workspace_size(int32_t batch, int32_t heads, int32_t capacity,
                                       size_t* bytes);
int tf_attention_decode(const void* qkv, int32_t batch, int32_t heads, int32_t head_dim,
                        const void* q_norm, const void* k_norm, float eps, float rope_theta,
                        const int32_t* positions, int32_t max_length, void* k_cache,
                        void* v_cache, int32_t capacity, float scale, int act, void* out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* model and session                                                          */

/* OLMoE geometry; NativeModelConfig (overlays/executorch/backends/mlx/runtime/
 * resident_prefill.h:18-42) as admitted for OLMoE by
 * NativeGraniteMoEPrefill::validate_config (MLXNativeGraniteMoEPrefill.h:306-330). */
typedef struct tf_olmoe_config {
  int32_t layers;
  int32_t hidden;
  int32_t heads;
  int32_t kv_heads;
  int32_t head_dim;
  int32_t intermediate;
  int32_t vocab;
  int32_t experts;
  int32_t top_k;
  int32_t capacity;
  float rms_eps;
  float rope_theta;
  int32_t act;
} tf_olmoe_config;

typedef struct tf_model tf_model;
typedef struct tf_session tf_session;

/* Device-resident model: one upload of every tensor, bound by its checkpoint
 * name ("model.layers.3.mlp.switch_mlp.up_proj.scales", "lm_head.weight", ...).
 * Replaces the NativeGraniteMoEPrefill constructor's name binding
 * (MLXNativeGraniteMoEPrefill.h:157-304). */
int tf_model_create(const tf_olmoe_config* config, int device, tf_model** model);
/* Copy `bytes` from `data` (host memory unless data_on_device) into the role
 * `name`; the copy has completed when the call returns, so the source may be
 * reused at once.  Unknown names, wrong sizes and rebinding are errors. */
int tf_model_bind(tf_model* model, const char* name, const void* data, size_t bytes,
                  int data_on_device);
/* All roles bound?  TF_ERR_STATE names the first missing role. */
int tf_model_finalize(tf_model* model);
int tf_model_destroy(tf_model* model);

/* Per-request fp16 KV cache for up to max_batch requests of `capacity`
 * slots, plus scratch for up to max(max_batch, max_prefill_tokens) rows per
 * call, all allocated here once.
 * Replaces MLXSequenceCache / Pool (patches/executorch.patch:1834-2094,
 * 2095-3566) and the resident session's owner (src/apple/
 * TFETResidentSession.mm:330-388). */
int tf_session_create(tf_model* model, int32_t max_batch, int32_t capacity,
                      int32_t max_prefill_tokens, tf_session** session);
int tf_session_destroy(tf_session* session);
/* Device pointers of one layer's caches, f16 [max_batch][kv_heads][capacity][head_dim]. */
int tf_session_kv(tf_session* session, int32_t layer, void** k_cache, void** v_cache);
/* Committed length of each request (host arrays of `batch` entries). */
int tf_session_set_lengths(tf_session* session, const int32_t* lengths, int32_t batch);
int tf_session_get_lengths(tf_session* session, int32_t* lengths, int32_t batch);

#define TF_HOST_INPUTS 1  /* token ids are host pointers                   */
#define TF_HOST_OUTPUT 2  /* logits / next-token output is a host pointer  */

/* Greedy next tokens: tokens[r] = all(isfinite(logits[r])) ? argmax(logits[r])
 * : -1 (int64, device memory), argmax taking the lowest index among equal
 * maxima; logits f32 [rows][vocab] in device memory.
 * Replaces the greedy submission's where(all(isfinite(logits)),
 * argmax(logits), -1) (patches/executorch.patch:1350-1353). */
int tf_greedy_tokens(const float* logits, int64_t rows, int64_t vocab, int64_t* tokens, void* stream);

/* One decode token for each of `batch` requests (requests 0..batch-1).
 * positions (always a host array, or NULL for "the committed lengths") must
 * equal each request's committed length; on success each length grows by
 * one.  token_ids are host or device memory per TF_HOST_INPUTS; logits
 * f32 [batch][vocab] (act-rounded values) per TF_HOST_OUTPUT.  With a host
 * output the call returns after the copy completes.
 * Replaces forwardTokenIDs:positions:nativeConfiguration: (include/trifuse/
 * apple/TFETResidentSession.h:354-359) -> NativeGraniteMoEPrefill::run with T=1
 * (MLXNativeGraniteMoEPrefill.h:347-493). */
int tf_session_decode(tf_session* session, const int64_t* token_ids, const int32_t* positions,
                      int32_t batch, float* logits, int flags, void* stream);

/* tf_session_decode followed by greedy selection on the device: tokens[b] =
 * all(isfinite(logits[b])) ? argmax : -1 (int64; device memory, or host
 * memory with TF_HOST_OUTPUT, in which case the call returns after the copy).
 * logits (optional, may be NULL) receives the f32 logits like
 * tf_session_decode.  Device-memory token_ids may be the `tokens` of the
 * previous greedy step, so step t+1 can be submitted before the host reads
 * step t's token (one-ahead submission); a negative id is read as token 0
 * (the reference's maximum(token, 0)) and the caller rejects the -1 it reads.
 * Host token ids must lie in [0, vocab).
 * Replaces nextGreedyPipelineExpectedGeneration: (src/apple/
 * TFETResidentSession.mm:1113-1189) and the resident greedy submission
 * (patches/executorch.patch:1341-1375, 1119-1127). */
int tf_session_decode_greedy(tf_session* session, const int64_t* token_ids, const int32_t* positions,
                             int32_t batch, int64_t* tokens, float* logits, int flags, void* stream);

/* Prefill a batch of requests: request requests[i] receives token_counts[i]
 * ids (concatenated in token_ids) starting at its committed length.  Writes
 * each request's last-token logits (f32 [num_requests][vocab]) unless
 * last_logits is NULL (cache-only).  Lengths grow by the counts.
 * Replaces prefillTokenIDs:nativeConfiguration: (TFETResidentSession.h:442-446)
 * -> NativeGraniteMoEPrefill::run with T > 1. */
int tf_session_prefill(tf_session* session, const int32_t* requests, const int32_t* token_counts,
                       int32_t num_requests, const int64_t* token_ids, float* last_logits,
                       int flags, void* stream);

/* Prefill of one request's prompt in chunks of chunk_tokens (<= the
 * session's max_prefill_tokens): every token id (host memory,
 * TF_HOST_INPUTS required) is checked against the vocabulary before the
 * first chunk runs; intermediate chunks only extend the KV cache, the last
 * one also writes the last row's logits (f32 [vocab], host or device per
 * TF_HOST_OUTPUT; a host copy containing a non-finite logit returns
 * TF_ERR_STATE).  Cancellation is honoured between chunks.  On an error the
 * chunks already run stay in the cache (tf_session_get_lengths tells).
 * Replaces prefillTokenIDs:nativeConfiguration:'s chunk loop (src/apple/
 * TFETResidentSession.mm:1546-1645: cache-only intermediate chunks, final
 * chunk with logits, finite check). */
int tf_session_prefill_chunked(tf_session* session, int32_t request, const int64_t* token_ids, int64_t count,
                               int32_t chunk_tokens, float* last_logits, int flags, void* stream);

/* Decode steps as CUDA graphs (default on): the first step of a shape
 * (batch, with/without logits, KV length rounded up to 256, QMM path) runs
 * eagerly, the second is captured on a session-owned stream, later ones
 * replay it, ordered after and before the caller's stream by events.  Host
 * inputs are copied before each replay; cancellation is checked before it.
 * Tracing runs steps eagerly.  The reference's counterpart is its resident
 * decode loop reusing the compiled MLX graph (patches/executorch.patch:
 * 1341-1375). */
int tf_session_graphs(tf_session* session, int enable);

/* Phase tracing (replaces the env-gated TRIFUSE_PREFILL_TIMING stderr lines,
 * src/apple/TFETResidentSession.mm:48-76, with device timing): while enabled,
 * each forward phase (embed, input_norm, qkv_proj, attention, o_proj,
 * post_norm, moe_router, moe_sort, moe_gate_up, moe_down, moe_combine,
 * final_norm, lm_head) is bracketed by CUDA events on the call's stream.
 * tf_session_trace_read synchronizes, returns per-phase total milliseconds
 * and bracket counts over all traced calls (arrays of tf_trace_phases()
 * entries), and clears the record. */
int tf_trace_phases(void);
const char* tf_trace_phase_name(int phase);
int tf_session_trace(tf_session* session, int enable);
int tf_session_trace_read(tf_session* session, float* total_ms, int32_t* counts);

/* Diagnostic capture: while `indices` or `hidden` is non-NULL, every forward
 * of at most max_rows rows writes each layer's top-k expert ids (int32
 * [layers][rows][top_k]) and output hidden states (act [layers][rows]
 * [hidden]) into them, with the rows of that call in order; in the last
 * layer of a prefill only each request's last row runs the MoE block, so
 * that layer's first rows hold them.  Decode steps then run without graph
 * replay.  Both NULL turns it off.  The counterpart of the reference's
 * inspect / receipt diagnostics (src/apple/TFETResidentSession.mm:1816-1967);
 * tests use it to check every layer against a CPU re-computation that starts
 * from the device's own state. */
int tf_session_capture(tf_session* session, int32_t* indices, void* hidden, int64_t max_rows);

/* Cooperative cancellation: the next layer boundary of a running or future
 * call returns TF_ERR_CANCELLED (TFETResidentSession.h:5-11).  A call
 * cancelled before it dispatched anything leaves the session as it was; one
 * cancelled between layers invalidates it (below). */
int tf_session_cancel(tf_session* session);

/* Dispatched failures.  Any failure after a session call has submitted work
 * (a launch or CUDA error, a cancellation between layers, or a device-side
 * failure found at a completion point) invalidates the session: the call
 * waits for the submitted work, returns the error, and every later call but
 * tf_session_kv / tf_session_get_lengths / tf_session_reset returns
 * TF_ERR_STATE.  Failures found by the checks before dispatch change nothing.
 * (TFETResidentSession.mm:388-392 quarantine and :667 failDispatched;
 * patches/executorch.patch:1486-1499 maps the failure to Error::Internal.)
 * Device-side failures are: a tensor-core pipeline wait that expired
 * (TF_ERR_TIMEOUT; the kernel gave up and its outputs are incomplete), an
 * activation beyond the f16 range reaching a tensor-core operand, and a
 * token id past the embedding table (both TF_ERR_STATE).  Calls with host
 * outputs and every prefill check for them before returning; calls with
 * device outputs do not wait for the device, so their failures surface at
 * the next such completion point or at tf_session_check. */
/* Completion point for device-output calls: waits for `stream`, then
 * reports (and invalidates the session on) a device-side failure since the
 * last check.  The reference's counterpart is its synchronize_storage +
 * finite check after submission (TFETResidentSession.mm:1612-1626). */
int tf_session_check(tf_session* session, void* stream);
/* Clear the cancellation flag and every request's length (beginRequest),
 * and re-admit an invalidated session (after waiting for the device and
 * clearing its device-side error flags). */
int tf_session_reset(tf_session* session);

/* Test hook: the number of SM clock cycles a tensor-core pipeline wait may
 * take before the kernel records TF_ERR_TIMEOUT and returns (cycles <= 0
 * restores the default, about one second), on the calling thread's current
 * device.  For failure-path tests; no reference counterpart. */
int tf_set_wait_limit(int64_t cycles);

#ifdef __cplusplus
}
#endif

#endif /* TRIFUSE_B200_H */
