// Host-side launcher interface shared by the C ABI (capi.cu), the model
// (model.cu) and the kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "../../include/trifuse_b200.h"

namespace tf {

// ---------------------------------------------------------------- errors
tf_status set_error(tf_status status, const char* fmt, ...);
void clear_error();
tf_status check_launch(const char* what);
// Kernels launched so far (the tf_launch_count counter); graph replays add
// the number of kernels they hold.
uint64_t launch_count();
void add_launches(int64_t n);

#define TF_TRY(expr)                          \
  do {                                        \
    tf_status _s = (expr);                    \
    if (_s != TF_OK) return _s;               \
  } while (0)

#define TF_CUDA(expr)                                                          \
  do {                                                                         \
    cudaError_t _e = (expr);                                                   \
    if (_e != cudaSuccess)                                                     \
      return ::tf::set_error(TF_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(_e)); \
  } while (0)

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Kernel attributes (cudaFuncSetAttribute) belong to the kernel's image on
// the current device, so a launcher sets them once per device: one bit per
// device ordinal below 64 (higher ordinals set them on every launch).
struct PerDeviceOnce {
  std::atomic<uint64_t> bits{0};
  // True when the current device (written to *dev) still needs the setup.
  bool needed(int* dev) {
    int d = 0;
    cudaGetDevice(&d);
    *dev = d;
    return d >= 64 || !((bits.load(std::memory_order_acquire) >> d) & 1u);
  }
  void mark(int dev) {
    if (dev < 64) bits.fetch_or(uint64_t(1) << dev, std::memory_order_release);
  }
};

// ---------------------------------------------------------------- tracing
// Phases of one forward; a session with profiling on records a CUDA event
// pair around each phase on the launching stream.
enum Phase {
  PH_EMBED = 0, PH_INPUT_NORM, PH_QKV, PH_ATTENTION, PH_O_PROJ, PH_POST_NORM, PH_ROUTER, PH_SORT,
  PH_GATE_UP, PH_DOWN, PH_COMBINE, PH_FINAL_NORM, PH_LM_HEAD, PH_COUNT
};
extern const char* const kPhaseNames[PH_COUNT];
struct Tracer {
  virtual void mark(int phase, bool begin, cudaStream_t s) = 0;
  virtual ~Tracer() = default;
};
// Tracer of the current call on this thread (nullptr = off).
extern thread_local Tracer* g_tracer;
inline void trace(int phase, bool begin, cudaStream_t s) {
  if (g_tracer) g_tracer->mark(phase, begin, s);
}
// Kernels launched by this library since load (all threads).
void count_launch();

// Bump allocator over a caller-provided workspace.
struct Carve {
  char* base;
  size_t cap;
  size_t used = 0;
  Carve(void* b, size_t c) : base(static_cast<char*>(b)), cap(c) {}
  template <typename P>
  P* take(size_t bytes) {
    used = align_up(used, 256);
    P* p = reinterpret_cast<P*>(base ? base + used : nullptr);
    used += bytes;
    return p;
  }
  bool ok() const { return used <= cap; }
};

inline int act_bytes(int dtype) { return dtype == TF_DTYPE_F32 ? 4 : 2; }
inline bool act_ok(int dtype) { return dtype == TF_DTYPE_F16 || dtype == TF_DTYPE_BF16; }

// ---------------------------------------------------------------- norm
tf_status launch_rms_norm(const void* x, int64_t rows, int width, const void* w, float eps,
                          int act, void* y, cudaStream_t s);
tf_status launch_embedding(const int64_t* ids, int64_t n, const tf_affine_weight& t, int out,
                           void* y, cudaStream_t s);

// ---------------------------------------------------------------- router
// Route-sort outputs for the router to produce itself (decode-sized
// batches): the last token's cluster to finish sorts every route in one CTA.
// arrivals: an int that is zero before the launch (left zero after it).
struct RouteSortOut {
  int32_t* order = nullptr;
  int32_t* inverse = nullptr;
  int32_t* offsets = nullptr;
  int32_t* active = nullptr;
  int32_t* active_count = nullptr;
  int* arrivals = nullptr;
};
// With `sort` the router also sorts the routes when it can (*sorted = true);
// otherwise the caller runs launch_route_sort.
tf_status launch_router(const void* x, int64_t tokens, int hidden, const tf_router_weight& r,
                        int experts, int k, int act, void* logits, int32_t* idx, void* gates,
                        cudaStream_t s, const RouteSortOut* sort = nullptr, bool* sorted = nullptr);
tf_status launch_route(const void* logits, int64_t tokens, int experts, int k, int act,
                       void* probs, int32_t* idx, void* gates, cudaStream_t s);
tf_status launch_topk(const void* probs, int64_t rows, int experts, int k, int act,
                      int32_t* idx, cudaStream_t s);
tf_status launch_take_along(const void* x, int64_t rows, int width, const int32_t* idx, int k,
                            int act, void* out, cudaStream_t s);

// Stable counting sort of n expert ids.  Outputs order/inverse [n],
// offsets [E+1], active [E] (ids of experts with routes, ascending) and
// active_count [1].  Workspace from sort_workspace_bytes.
size_t sort_workspace_bytes(int64_t n, int experts);
tf_status launch_route_sort(const int32_t* ids, int64_t n, int experts, int32_t* order,
                            int32_t* inverse, int32_t* offsets, int32_t* active,
                            int32_t* active_count, void* ws, size_t ws_bytes, cudaStream_t s);
// dst[i] = src[perm[i]] / div
tf_status launch_gather_index(const int32_t* src, const int32_t* perm, int64_t n, int div,
                              int32_t* dst, cudaStream_t s);

// ---------------------------------------------------------------- 4-bit QMM
enum QmmMode { QMM_DENSE = 0, QMM_GROUPED = 1, QMM_PER_ROUTE = 2 };
// EPI_F32: y is float and holds the act-rounded result (fp32 logits).
enum QmmEpilogue { EPI_PLAIN = 0, EPI_SWIGLU = 1, EPI_RESIDUAL = 2, EPI_F32 = 3 };

struct QmmProblem {
  int mode = QMM_DENSE;
  int epilogue = EPI_PLAIN;
  int act = TF_DTYPE_F16;
  // input rows: slot n reads x row  x_index ? x_index[n] / x_div : n / rows_per_x
  const void* x = nullptr;
  int64_t x_stride = 0;
  const int32_t* x_index = nullptr;
  int x_div = 1;
  int rows_per_x = 1;
  int64_t n = 0;  // slots (output rows)
  // QMM_PER_ROUTE: expert of slot n; QMM_GROUPED: offsets/active/active_count
  const int32_t* indices = nullptr;
  const int32_t* offsets = nullptr;
  const int32_t* active = nullptr;
  const int32_t* active_count = nullptr;
  // weights: w0 (and w1 = up projection for EPI_SWIGLU, w0 = gate)
  tf_affine_weight w0{};
  tf_affine_weight w1{};
  // output
  void* y = nullptr;
  int64_t y_stride = 0;
  // EPI_PLAIN: output row of slot n is y_index[n] (NULL: n), so a grouped
  // problem can write its rows back in the caller's route order.
  const int32_t* y_index = nullptr;
  const void* residual = nullptr;  // EPI_RESIDUAL, indexed like y
  int64_t residual_stride = 0;
  // Tensor-core operand: an f16 copy of the activations with contiguous rows
  // (dense bf16: x converted, same stride; grouped: slot-ordered rows of
  // width in_features).  x16_perm: the copy holds each group of 8 columns in
  // the order [0,4,1,5,2,6,3,7] (the tensor-core dequant's own order).
  const void* x16 = nullptr;
  int x16_perm = 0;
  // EPI_SWIGLU: y is written in f16 in the x16_perm order, as the operand of
  // a following tensor-core QMM.
  int y_f16 = 0;
  // Optional buffers of the tensor-core split schedule (decode-sized tiles
  // spread evenly over every SM): fp32 partials of at least
  // qmm_split_partial_bytes() and counter_cap int counters that are zero when
  // the launch starts (a completed launch leaves them zero again).  Without
  // them each block takes whole tiles.
  float* partials = nullptr;
  size_t partial_bytes = 0;
  int* counters = nullptr;
  int64_t counter_cap = 0;
};
// Bytes of fp32 partials the tensor-core split schedule needs on this device.
size_t qmm_split_partial_bytes();
// Counters of the split schedule in a workspace (four per tile).
constexpr int64_t kQmmSplitCounters = 16384;
// Path launch_qmm would take for this problem (true = tensor cores).
bool qmm_uses_tc(const QmmProblem& p);
// f16 copy of n bf16 values (rows of 2048), optionally in the x16_perm order.
tf_status launch_bf16_to_f16(const void* x, int64_t n, void* y, int permute, cudaStream_t s);
// y[i][:] = f16(x[perm ? perm[i] / div : i][:]) for i < rows (tensor-core
// operand), optionally in the x16_perm column order.
tf_status launch_gather_f16(const void* x, int64_t x_stride, int act, const int32_t* perm, int div, int64_t rows,
                            int width, void* y, int permute, cudaStream_t s);
// Dispatches to the tensor-core kernel (launch_qmm_tc) when the problem has
// enough tokens per weight matrix, else to the CUDA-core GEMV.
tf_status launch_qmm(const QmmProblem& p, cudaStream_t s);
tf_status launch_qmm_gemv(const QmmProblem& p, cudaStream_t s);
tf_status launch_qmm_tc(const QmmProblem& p, cudaStream_t s);
// 0 = automatic, 1 = CUDA-core GEMV only, 2 = tensor cores whenever eligible.
extern int g_qmm_path;
int read_tc_error(bool clear);
// Cycles a tensor-core pipeline wait may take (<= 0: the default), current device.
tf_status set_wait_limit(long long cycles);
// Device addresses of the tensor-core error code and wait limit, for
// kernels in other translation units that record into the same flag.
tf_status tc_flags(int** error, long long** wait_cycles);
int read_embed_error(bool clear);
// tokens[r] = all(isfinite(logits[r])) ? argmax (lowest index on ties) : -1.
tf_status launch_greedy(const float* logits, int64_t rows, int64_t vocab, int64_t* tokens, cudaStream_t s);

// y[i][:] = x[idx[i] / div][:] for i < n (act rows of `width`, width % 8 == 0).
tf_status launch_gather_rows(const void* x, int64_t x_stride, const int32_t* idx, int div, int64_t n, int width,
                             int act, void* y, cudaStream_t s);

// ---------------------------------------------------------------- combine
// With norm_out, also norm_out = RMSNorm(out) * norm_w (the next layer's
// input norm, in rms_norm_kernel's order, bit-identical to it).
tf_status launch_combine(const void* y_sorted, const int32_t* inverse, const void* gates,
                         const void* residual, int64_t tokens, int k, int hidden, int act,
                         void* out, cudaStream_t s, const void* norm_w = nullptr, float eps = 0.f,
                         void* norm_out = nullptr);

// ---------------------------------------------------------------- MoE block
// with_split adds the tensor-core split buffers (about 10 MB).
size_t moe_workspace_bytes(const tf_moe_args* a, bool with_split = true);
// Runs the block on a workspace of at least moe_workspace_bytes(a, false),
// with the split schedule when it holds moe_workspace_bytes(a, true).
// counters_zero: the workspace's split counters are known to be zero.
// The next layer's input RMSNorm fused into the block's combine.
struct MoeNextNorm {
  const void* w = nullptr;
  float eps = 0.f;
  void* out = nullptr;
};
tf_status moe_run(const tf_moe_args* a, void* ws, size_t ws_bytes, cudaStream_t s, bool counters_zero = false,
                  const MoeNextNorm* next = nullptr);

// ---------------------------------------------------------------- attention
// Row r (one query token) of request req[r] (r when req == NULL) at absolute
// position pos[r]: append its k/v at slot pos[r], attend slots 0..pos[r].
struct AttnProblem {
  const void* qkv = nullptr;  // act [rows][3 * heads * head_dim]
  int64_t rows = 0;
  int heads = 0;
  int head_dim = 0;
  const void* q_norm = nullptr;  // f16 [heads * head_dim]
  const void* k_norm = nullptr;
  float eps = 1e-5f;
  float theta = 10000.f;
  // Optional: (cos, sin) of every position below capacity, [capacity][64]
  // float2 from launch_rope_table with the same theta (bit-identical to the
  // kernel's own sincosf).
  const void* rope = nullptr;
  // The workspace's split-arrival counters are zero (a session's workspace,
  // cleared once and left zero by every launch); else they are cleared.
  bool arrivals_zero = false;
  int64_t ws_rows = 0;  // rows the workspace was sized for (attention_ws_bytes); 0: rows
  const int32_t* pos = nullptr;  // device [rows]
  const int32_t* req = nullptr;  // device [rows] or NULL
  int max_len = 0;               // >= pos[r] + 1 for every row (host bound)
  void* k_cache = nullptr;       // f16 [requests][heads][capacity][head_dim]
  void* v_cache = nullptr;
  int capacity = 0;
  float scale = 1.f;
  int act = TF_DTYPE_F16;
  void* out = nullptr;  // act [rows][heads * head_dim]
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // Optional (prefill): device int4 {first row, rows <= kPrefillQueryBlock,
  // request, first position} per query block; every row of a block belongs
  // to one request and the rows' positions are consecutive.  With it the
  // attention runs the tiled tensor-core kernel instead of the per-row
  // split-K one; cache_requests (the caches' first dimension) bounds its
  // tile copies.
  const int4* qblocks = nullptr;
  int nqblocks = 0;
  int cache_requests = 0;
  // Optional: attend only the rows qrows[0..nq) (device), writing output row
  // i for qrows[i]; every row is still appended.  nq == 0: append only.
  const int32_t* qrows = nullptr;
  int64_t nq = 0;
};
constexpr int kPrefillQueryBlock = 256;
size_t attention_ws_bytes(int64_t rows, int heads, int capacity, int act);
tf_status launch_attn_prefill_tc(const AttnProblem& a, const void* q, cudaStream_t s);
tf_status launch_rope_table(float theta, int positions, void* tab, cudaStream_t s);
tf_status launch_attention(const AttnProblem& a, cudaStream_t s);

}  // namespace tf
