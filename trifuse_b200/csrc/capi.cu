// C ABI: argument validation and orchestration of the operator entry points.
// Validation mirrors the reference's admission checks (validate_affine,
// overlays/executorch/backends/mlx/native_affine_ops.py:12-26, and the
// adapter's need() checks, MLXNativeGraniteMoEPrefill.h:220-262, 306-330)
// and always runs before any launch.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace tf {

static thread_local std::string g_error;

tf_status set_error(tf_status status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
  return status;
}

void clear_error() { g_error.clear(); }

static std::atomic<uint64_t> g_launches{0};
thread_local Tracer* g_tracer = nullptr;
const char* const kPhaseNames[PH_COUNT] = {"embed", "input_norm", "qkv_proj", "attention", "o_proj",
                                           "post_norm", "moe_router", "moe_sort", "moe_gate_up",
                                           "moe_down", "moe_combine", "final_norm", "lm_head"};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
uint64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }
void add_launches(int64_t n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

tf_status check_launch(const char* what) {
  count_launch();
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(TF_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return TF_OK;
}

bool kernel_image_ok();

}  // namespace tf

using namespace tf;

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

tf_status check_act(int act) {
  if (!act_ok(act)) return set_error(TF_ERR_INVALID_ARGUMENT, "activation dtype must be f16 or bf16");
  return TF_OK;
}

// validate_affine (native_affine_ops.py:12-26) for the 4-bit/group-64 form.
tf_status check_affine(const tf_affine_weight* w, const char* what, bool stacked) {
  if (!w) return set_error(TF_ERR_INVALID_ARGUMENT, "%s: weight descriptor is NULL", what);
  if (!(w->bits == 4 || w->bits == 8) ||
      !(w->group_size == 32 || w->group_size == 64 || w->group_size == 128))
    return set_error(TF_ERR_INVALID_ARGUMENT, "%s: Native affine requires bits4/8 and group32/64/128", what);
  if (w->bits != 4 || w->group_size != 64)
    return set_error(TF_ERR_UNSUPPORTED, "%s: only affine bits 4 / group 64 runs on this path", what);
  if (w->out_features <= 0 || w->in_features <= 0 || (stacked ? w->experts <= 0 : w->experts > 1) ||
      w->experts < 0)
    return set_error(TF_ERR_SHAPE, "%s: Native affine packed/group dimensions differ", what);
  if (w->in_features % w->group_size)
    return set_error(TF_ERR_SHAPE, "%s: Native affine packed/group dimensions differ", what);
  if (!w->q || !w->scales || !w->biases)
    return set_error(TF_ERR_INVALID_ARGUMENT, "%s: NULL Q/S/B pointer", what);
  if (!aligned16(w->q)) return set_error(TF_ERR_INVALID_ARGUMENT, "%s: Q must be 16-byte aligned", what);
  return TF_OK;
}

cudaStream_t st(void* s) { return reinterpret_cast<cudaStream_t>(s); }

}  // namespace

extern "C" {

int tf_abi_version(void) { return TF_ABI_VERSION; }

uint64_t tf_launch_count(void) { return g_launches.load(); }

int tf_set_qmm_path(int path) {
  if (path < 0 || path > 2) return set_error(TF_ERR_INVALID_ARGUMENT, "qmm path must be 0, 1 or 2");
  g_qmm_path = path;
  return TF_OK;
}

int tf_set_wait_limit(int64_t cycles) { return set_wait_limit(cycles); }

int tf_device_error(int clear) {
  TF_CUDA(cudaDeviceSynchronize());
  const int tc = read_tc_error(clear != 0);
  const int emb = read_embed_error(clear != 0);
  return tc ? tc : emb;
}

const char* tf_last_error(void) { return g_error.c_str(); }

const char* tf_status_name(int status) {
  switch (status) {
    case TF_OK: return "TF_OK";
    case TF_ERR_INVALID_ARGUMENT: return "TF_ERR_INVALID_ARGUMENT";
    case TF_ERR_SHAPE: return "TF_ERR_SHAPE";
    case TF_ERR_OUT_OF_MEMORY: return "TF_ERR_OUT_OF_MEMORY";
    case TF_ERR_CUDA: return "TF_ERR_CUDA";
    case TF_ERR_NCCL: return "TF_ERR_NCCL";
    case TF_ERR_TIMEOUT: return "TF_ERR_TIMEOUT";
    case TF_ERR_CANCELLED: return "TF_ERR_CANCELLED";
    case TF_ERR_UNSUPPORTED: return "TF_ERR_UNSUPPORTED";
    case TF_ERR_STATE: return "TF_ERR_STATE";
    case TF_ERR_CAPACITY: return "TF_ERR_CAPACITY";
    default: return "TF_ERR_UNKNOWN";
  }
}

int tf_device_check(int device) {
  int n = 0;
  TF_CUDA(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return set_error(TF_ERR_INVALID_ARGUMENT, "no CUDA device %d", device);
  cudaDeviceProp prop;
  TF_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return set_error(TF_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a",
                     device, prop.major, prop.minor);
  int prev = 0;
  TF_CUDA(cudaGetDevice(&prev));
  TF_CUDA(cudaSetDevice(device));
  const bool ok = kernel_image_ok();
  TF_CUDA(cudaSetDevice(prev));
  if (!ok) return set_error(TF_ERR_UNSUPPORTED, "sm_100a kernels do not load on device %d", device);
  return TF_OK;
}

int tf_rms_norm(const void* x, int64_t rows, int32_t width, const void* weight, float eps, int act,
                void* y, void* stream) {
  TF_TRY(check_act(act));
  if (rows < 0 || width <= 0 || width % 256 || width > 8192)
    return set_error(TF_ERR_SHAPE, "rms_norm: width must be a multiple of 256 up to 8192");
  if (!(eps > 0)) return set_error(TF_ERR_INVALID_ARGUMENT, "rms_norm: eps must be positive");
  if (rows && (!x || !weight || !y || !aligned16(x) || !aligned16(weight) || !aligned16(y)))
    return set_error(TF_ERR_INVALID_ARGUMENT, "rms_norm: NULL or unaligned pointer");
  return launch_rms_norm(x, rows, width, weight, eps, act, y, st(stream));
}

int tf_affine_qmm(const void* x, int64_t rows, const tf_affine_weight* w, int act, void* y,
                  void* stream) {
  TF_TRY(check_act(act));
  TF_TRY(check_affine(w, "qmm", false));
  if (rows < 0) return set_error(TF_ERR_SHAPE, "qmm: negative rows");
  if (rows && (!x || !y || !aligned16(x)))
    return set_error(TF_ERR_INVALID_ARGUMENT, "qmm: NULL or unaligned activation pointer");
  QmmProblem p;
  p.mode = QMM_DENSE;
  p.act = act;
  p.x = x;
  p.x_stride = w->in_features;
  p.n = rows;
  p.w0 = *w;
  p.y = y;
  p.y_stride = w->out_features;
  return launch_qmm(p, st(stream));
}

int tf_affine_gather_qmm(const void* x, int64_t x_rows, int32_t rows_per_x, const int32_t* x_index,
                         const int32_t* indices, int64_t n, const tf_affine_weight* w,
                         int sorted_indices, int act, void* y, void* stream) {
  (void)sorted_indices;
  TF_TRY(check_act(act));
  TF_TRY(check_affine(w, "gather_qmm", true));
  if (n < 0 || x_rows < 0 || (!x_index && rows_per_x <= 0))
    return set_error(TF_ERR_SHAPE, "gather_qmm: Native affine expert input differs");
  if (!x_index && n > 0 && (n - 1) / rows_per_x >= x_rows)
    return set_error(TF_ERR_SHAPE, "gather_qmm: broadcast rows exceed x");
  if (n && (!x || !y || !indices || !aligned16(x)))
    return set_error(TF_ERR_INVALID_ARGUMENT, "gather_qmm: NULL or unaligned pointer");
  QmmProblem p;
  p.mode = QMM_PER_ROUTE;
  p.act = act;
  p.x = x;
  p.x_stride = w->in_features;
  p.x_index = x_index;
  p.rows_per_x = rows_per_x > 0 ? rows_per_x : 1;
  p.n = n;
  p.indices = indices;
  p.w0 = *w;
  p.y = y;
  p.y_stride = w->out_features;
  return launch_qmm(p, st(stream));
}

int tf_moe_combine(const void* y_sorted, const int32_t* inverse, const void* gates, const void* residual,
                   int64_t tokens, int32_t k, int32_t hidden, int act, void* out, void* stream) {
  TF_TRY(check_act(act));
  if (tokens < 0 || k <= 0 || hidden <= 0 || hidden % 8)
    return set_error(TF_ERR_SHAPE, "combine: tokens %lld k %d hidden %d", (long long)tokens, k, hidden);
  if (tokens && (!y_sorted || !inverse || !gates || !residual || !out || !aligned16(y_sorted) ||
                 !aligned16(residual) || !aligned16(out)))
    return set_error(TF_ERR_INVALID_ARGUMENT, "combine: NULL or unaligned pointer");
  return launch_combine(y_sorted, inverse, gates, residual, tokens, k, hidden, act, out, st(stream));
}

int tf_greedy_tokens(const float* logits, int64_t rows, int64_t vocab, int64_t* tokens, void* stream) {
  if (rows < 0 || vocab <= 0) return set_error(TF_ERR_SHAPE, "greedy: rows %lld vocab %lld", (long long)rows,
                                               (long long)vocab);
  if (rows && (!logits || !tokens)) return set_error(TF_ERR_INVALID_ARGUMENT, "greedy: NULL pointer");
  return launch_greedy(logits, rows, vocab, tokens, st(stream));
}

int tf_affine_embedding(const int64_t* ids, int64_t n, const tf_affine_weight* table, int out_dtype,
                        void* y, void* stream) {
  TF_TRY(check_act(out_dtype));
  TF_TRY(check_affine(table, "embedding", false));
  if (n < 0) return set_error(TF_ERR_SHAPE, "embedding: negative count");
  if (n && (!ids || !y || !aligned16(y)))
    return set_error(TF_ERR_INVALID_ARGUMENT, "embedding: NULL or unaligned pointer");
  return launch_embedding(ids, n, *table, out_dtype, y, st(stream));
}

static tf_status check_route(int64_t rows, int32_t experts, int32_t k) {
  if (rows < 0 || experts <= 0 || experts > 64)
    return set_error(TF_ERR_SHAPE, "OLMoE router geometry differs (experts must be 1..64)");
  if (k <= 0 || k > experts || k > 32) return set_error(TF_ERR_INVALID_ARGUMENT, "Invalid OLMoE top-k");
  return TF_OK;
}

int tf_olmoe_softmax(const void* logits, int64_t rows, int32_t experts, int act, void* probs,
                     void* stream) {
  TF_TRY(check_act(act));
  TF_TRY(check_route(rows, experts, 1));
  if (rows && (!logits || !probs)) return set_error(TF_ERR_INVALID_ARGUMENT, "softmax: NULL pointer");
  return launch_route(logits, rows, experts, 1, act, probs, nullptr, nullptr, st(stream));
}

int tf_olmoe_topk_indices(const void* probs, int64_t rows, int32_t experts, int32_t k, int act,
                          int32_t* indices, void* stream) {
  TF_TRY(check_act(act));
  TF_TRY(check_route(rows, experts, k));
  if (rows && (!probs || !indices)) return set_error(TF_ERR_INVALID_ARGUMENT, "topk: NULL pointer");
  return launch_topk(probs, rows, experts, k, act, indices, st(stream));
}

int tf_take_along_last(const void* x, int64_t rows, int32_t width, const int32_t* indices, int32_t k,
                       int act, void* out, void* stream) {
  TF_TRY(check_act(act));
  if (rows < 0 || width <= 0 || k < 0) return set_error(TF_ERR_SHAPE, "take_along_last: bad shape");
  if (rows && k && (!x || !indices || !out))
    return set_error(TF_ERR_INVALID_ARGUMENT, "take_along_last: NULL pointer");
  return launch_take_along(x, rows, width, indices, k, act, out, st(stream));
}

int tf_olmoe_route(const void* logits, int64_t tokens, int32_t experts, int32_t k, int act,
                   int32_t* indices, void* gates, void* stream) {
  TF_TRY(check_act(act));
  TF_TRY(check_route(tokens, experts, k));
  if (tokens && (!logits || !indices || !gates))
    return set_error(TF_ERR_INVALID_ARGUMENT, "route: NULL pointer");
  return launch_route(logits, tokens, experts, k, act, nullptr, indices, gates, st(stream));
}

static tf_status check_router(const tf_router_weight* r, int32_t hidden, int32_t experts) {
  if (!r) return set_error(TF_ERR_INVALID_ARGUMENT, "router weight is NULL");
  if (r->dense) {
    if (!aligned16(r->dense)) return set_error(TF_ERR_INVALID_ARGUMENT, "router: unaligned dense weight");
    return TF_OK;
  }
  TF_TRY(check_affine(&r->affine, "router", false));
  if (r->affine.out_features != experts || r->affine.in_features != hidden)
    return set_error(TF_ERR_SHAPE, "router: affine weight must be [experts][hidden]");
  return TF_OK;
}

int tf_olmoe_router(const void* x, int64_t tokens, int32_t hidden, const tf_router_weight* router,
                    int32_t experts, int32_t k, int act, void* logits, int32_t* indices, void* gates,
                    void* stream) {
  TF_TRY(check_act(act));
  TF_TRY(check_route(tokens, experts, k));
  TF_TRY(check_router(router, hidden, experts));
  if (hidden % 256 || hidden > 2048) return set_error(TF_ERR_SHAPE, "router: hidden must be a multiple of 256 <= 2048");
  if (tokens && (!x || !aligned16(x) || !indices || !gates))
    return set_error(TF_ERR_INVALID_ARGUMENT, "router: NULL or unaligned pointer");
  return launch_router(x, tokens, hidden, *router, experts, k, act, logits, indices, gates, st(stream));
}

// ---------------------------------------------------------------- route sort

static size_t sort_bundle_bytes(int64_t n, int32_t experts) {
  Carve c(nullptr, 0);
  c.take<int32_t>(experts * 4);       // active
  c.take<int32_t>(4);                 // active_count
  c.take<char>(sort_workspace_bytes(n, experts));
  return c.used;
}

int tf_moe_route_sort_workspace_size(int64_t tokens, int32_t k, int32_t experts, size_t* bytes) {
  if (!bytes || tokens < 0 || k <= 0 || experts <= 0) return set_error(TF_ERR_INVALID_ARGUMENT, "bad arguments");
  *bytes = sort_bundle_bytes(tokens * k, experts);
  return TF_OK;
}

int tf_moe_route_sort(const int32_t* indices, int64_t tokens, int32_t k, int32_t experts,
                      int32_t* order, int32_t* inverse, int32_t* offsets, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (tokens < 0 || k <= 0 || experts <= 0 || experts > 256 || tokens > INT32_MAX / k)
    return set_error(TF_ERR_SHAPE, "route sort: bad geometry");
  const int64_t n = tokens * k;
  if (!offsets || (n && (!indices || !order || !inverse)))
    return set_error(TF_ERR_INVALID_ARGUMENT, "route sort: NULL pointer");
  if (workspace_bytes < sort_bundle_bytes(n, experts) || !workspace)
    return set_error(TF_ERR_INVALID_ARGUMENT, "route sort: workspace too small");
  Carve c(workspace, workspace_bytes);
  int32_t* active = c.take<int32_t>(experts * 4);
  int32_t* active_count = c.take<int32_t>(4);
  void* sws = c.take<char>(sort_workspace_bytes(n, experts));
  return launch_route_sort(indices, n, experts, order, inverse, offsets, active, active_count, sws,
                           sort_workspace_bytes(n, experts), st(stream));
}

// ---------------------------------------------------------------- MoE block

struct MoePlan {
  void* logits;
  int32_t* idx;
  void* gates;
  int32_t* order;
  int32_t* inverse;
  int32_t* offsets;
  int32_t* active;
  int32_t* active_count;
  void* sort_ws;
  size_t sort_ws_bytes;
  void* h;
  void* y;
  // f16 tensor-core operand: x rows in slot order when gate/up runs on tensor cores, else the
  // f16 copy of h when only the down projection does (never both in one call).
  void* op16;
  // Split-schedule buffers of the tensor-core QMMs (NULL in the plan without them).
  float* partials;
  size_t partial_bytes;
  int* counters;
  size_t used;
};

// with_split: also carve the tensor-core split buffers (fp32 partials and
// tile counters) that spread decode-sized expert tiles over every SM.
static MoePlan plan_moe(const tf_moe_args* a, void* ws, size_t ws_bytes, bool with_split = true) {
  const int64_t T = a->tokens, N = a->tokens * a->top_k;
  const int ab = act_bytes(a->act);
  Carve c(ws, ws_bytes);
  MoePlan p;
  // The arrival counters (split tiles, route sort) come first, at an offset
  // that does not depend on the token count: a workspace reused by calls of
  // different sizes (a session's prefill, then its decode steps) finds them
  // where the last call left them at zero, never on another call's data.
  p.partials = nullptr;
  p.partial_bytes = 0;
  p.counters = nullptr;
  if (with_split) {
    p.counters = c.take<int>((size_t)(kQmmSplitCounters + 1) * sizeof(int));  // + the router's arrivals
    p.partial_bytes = qmm_split_partial_bytes();
    p.partials = c.take<float>(p.partial_bytes);
  }
  p.logits = a->logits ? a->logits : c.take<char>((size_t)T * a->experts * ab);
  p.idx = a->indices ? a->indices : c.take<int32_t>((size_t)N * 4);
  p.gates = a->gates ? a->gates : c.take<char>((size_t)N * ab);
  p.order = c.take<int32_t>((size_t)N * 4);
  p.inverse = c.take<int32_t>((size_t)N * 4);
  p.offsets = c.take<int32_t>((size_t)(a->experts + 1) * 4);
  p.active = c.take<int32_t>((size_t)a->experts * 4);
  p.active_count = c.take<int32_t>(4);
  p.sort_ws_bytes = sort_workspace_bytes(N, a->experts);
  p.sort_ws = c.take<char>(p.sort_ws_bytes);
  p.h = c.take<char>((size_t)N * a->intermediate * ab);
  p.y = c.take<char>((size_t)N * a->hidden * ab);
  p.op16 = c.take<char>((size_t)N * (a->hidden > a->intermediate ? a->hidden : a->intermediate) * 2);
  p.used = c.used;
  return p;
}

static tf_status check_moe(const tf_moe_args* a) {
  if (!a) return set_error(TF_ERR_INVALID_ARGUMENT, "moe: args is NULL");
  TF_TRY(check_act(a->act));
  TF_TRY(check_route(a->tokens, a->experts, a->top_k));
  if (a->tokens > INT32_MAX / a->top_k) return set_error(TF_ERR_SHAPE, "moe: more than 2^31 - 1 routes");
  if (a->hidden % 256 || a->hidden > 2048 || a->intermediate % 64 || a->intermediate <= 0)
    return set_error(TF_ERR_SHAPE, "moe: unsupported hidden/intermediate geometry");
  TF_TRY(check_router(&a->router, a->hidden, a->experts));
  TF_TRY(check_affine(&a->gate_proj, "gate_proj", true));
  TF_TRY(check_affine(&a->up_proj, "up_proj", true));
  TF_TRY(check_affine(&a->down_proj, "down_proj", true));
  const tf_affine_weight* g = &a->gate_proj;
  const tf_affine_weight* u = &a->up_proj;
  const tf_affine_weight* d = &a->down_proj;
  if (g->experts != a->experts || u->experts != a->experts || d->experts != a->experts ||
      g->out_features != a->intermediate || g->in_features != a->hidden ||
      u->out_features != a->intermediate || u->in_features != a->hidden ||
      d->out_features != a->hidden || d->in_features != a->intermediate)
    return set_error(TF_ERR_SHAPE, "moe: packed parameter geometry differs");
  if (a->tokens && (!a->x || !a->residual || !a->out || !aligned16(a->x) || !aligned16(a->residual) ||
                    !aligned16(a->out)))
    return set_error(TF_ERR_INVALID_ARGUMENT, "moe: NULL or unaligned activation pointer");
  return TF_OK;
}

// counters_zero: the caller guarantees the split counters are zero (a
// session's scratch, zeroed once and left zero by every completed launch);
// otherwise they are cleared first.
static tf_status run_moe(const tf_moe_args* a, const MoePlan& p, cudaStream_t s, bool counters_zero = false,
                         const MoeNextNorm* next = nullptr) {
  const int64_t N = a->tokens * a->top_k;
  if (p.counters && !counters_zero)
    TF_CUDA(cudaMemsetAsync(p.counters, 0, (size_t)(kQmmSplitCounters + 1) * sizeof(int), s));
  RouteSortOut so;
  so.order = p.order;
  so.inverse = p.inverse;
  so.offsets = p.offsets;
  so.active = p.active;
  so.active_count = p.active_count;
  so.arrivals = p.counters ? p.counters + kQmmSplitCounters : nullptr;
  bool sorted = false;
  trace(PH_ROUTER, true, s);
  TF_TRY(launch_router(a->x, a->tokens, a->hidden, a->router, a->experts, a->top_k, a->act,
                       p.logits, p.idx, p.gates, s, &so, &sorted));
  trace(PH_ROUTER, false, s);
  if (!sorted) {
    trace(PH_SORT, true, s);
    TF_TRY(launch_route_sort(p.idx, N, a->experts, p.order, p.inverse, p.offsets, p.active,
                             p.active_count, p.sort_ws, p.sort_ws_bytes, s));
    trace(PH_SORT, false, s);
  }
  QmmProblem up;
  up.mode = QMM_GROUPED;
  up.epilogue = EPI_SWIGLU;
  up.act = a->act;
  up.x = a->x;
  up.x_stride = a->hidden;
  up.x_index = p.order;
  up.x_div = a->top_k;
  up.n = N;
  up.offsets = p.offsets;
  up.active = p.active;
  up.active_count = p.active_count;
  up.w0 = a->gate_proj;
  up.w1 = a->up_proj;
  up.y = p.h;
  up.y_stride = a->intermediate;
  up.partials = p.partials;
  up.partial_bytes = p.partial_bytes;
  up.counters = p.counters;
  up.counter_cap = p.counters ? kQmmSplitCounters : 0;
  QmmProblem dn = up;
  dn.epilogue = EPI_PLAIN;
  dn.x = p.h;
  dn.x_stride = a->intermediate;
  dn.x_index = nullptr;
  dn.x_div = 1;
  dn.rows_per_x = 1;
  dn.w0 = a->down_proj;
  dn.y = p.y;
  dn.y_stride = a->hidden;
  const bool tc_up = qmm_uses_tc(up), tc_dn = qmm_uses_tc(dn);
  trace(PH_GATE_UP, true, s);
  if (tc_up) {
    // The tensor cores read the expert inputs as contiguous f16 rows in slot order.
    TF_TRY(launch_gather_f16(a->x, a->hidden, a->act, p.order, a->top_k, N, a->hidden, p.op16, 1, s));
    up.x16 = p.op16;
    up.x16_perm = 1;
    if (tc_dn) {  // h goes straight to the next tensor-core QMM in f16 storage
      up.y_f16 = 1;
      dn.x16 = p.h;
      dn.x16_perm = 1;
    }
  }
  TF_TRY(launch_qmm(up, s));
  trace(PH_GATE_UP, false, s);
  if (tc_dn && !up.y_f16) {
    TF_TRY(launch_gather_f16(p.h, a->intermediate, a->act, nullptr, 1, N, a->intermediate, p.op16, 1, s));
    dn.x16 = p.op16;
    dn.x16_perm = 1;
  }
  trace(PH_DOWN, true, s);
  TF_TRY(launch_qmm(dn, s));
  trace(PH_DOWN, false, s);
  trace(PH_COMBINE, true, s);
  TF_TRY(launch_combine(p.y, p.inverse, p.gates, a->residual, a->tokens, a->top_k, a->hidden, a->act,
                        a->out, s, next ? next->w : nullptr, next ? next->eps : 0.f, next ? next->out : nullptr));
  trace(PH_COMBINE, false, s);
  return TF_OK;
}

}  // extern "C"

namespace tf {
size_t moe_workspace_bytes(const tf_moe_args* a, bool with_split) { return plan_moe(a, nullptr, 0, with_split).used; }
tf_status moe_run(const tf_moe_args* a, void* ws, size_t ws_bytes, cudaStream_t s, bool counters_zero,
                  const MoeNextNorm* next) {
  if (a->tokens == 0) return TF_OK;
  const bool split = plan_moe(a, nullptr, 0, true).used <= ws_bytes;
  const MoePlan p = plan_moe(a, ws, ws_bytes, split);
  if (p.used > ws_bytes) return set_error(TF_ERR_INVALID_ARGUMENT, "moe: workspace too small");
  return run_moe(a, p, s, counters_zero, next);
}
}  // namespace tf

extern "C" {

int tf_moe_workspace_size(const tf_moe_args* args, size_t* bytes) {
  TF_TRY(check_moe(args));
  if (!bytes) return set_error(TF_ERR_INVALID_ARGUMENT, "bytes is NULL");
  *bytes = plan_moe(args, nullptr, 0).used;
  return TF_OK;
}

int tf_moe_forward(const tf_moe_args* args, void* workspace, size_t workspace_bytes, void* stream) {
  TF_TRY(check_moe(args));
  // The reported size includes the split buffers; a workspace of at least the
  // size without them still runs (every tile then goes to one block).
  const MoePlan full = plan_moe(args, nullptr, 0, true);
  const MoePlan need = plan_moe(args, nullptr, 0, false);
  if (workspace_bytes < need.used || (need.used && !workspace))
    return set_error(TF_ERR_INVALID_ARGUMENT, "moe: workspace %zu bytes < required %zu", workspace_bytes,
                     full.used);
  if (args->tokens == 0) return TF_OK;
  const MoePlan p = plan_moe(args, workspace, workspace_bytes, workspace_bytes >= full.used);
  return run_moe(args, p, st(stream));
}

// ---------------------------------------------------------------- expert hook

struct ExpertPlan {
  int32_t *order, *inverse, *xrow, *offsets, *active, *active_count;
  void *sws, *h, *x16, *h16;
  size_t sws_bytes, used;
};

static ExpertPlan plan_expert(void* ws, size_t ws_bytes, int64_t n, int64_t x_rows, int32_t hidden,
                              int32_t intermediate, int32_t experts, int act) {
  Carve c(ws, ws_bytes);
  ExpertPlan p;
  p.order = c.take<int32_t>((size_t)n * 4);
  p.inverse = c.take<int32_t>((size_t)n * 4);
  p.xrow = c.take<int32_t>((size_t)n * 4);
  p.offsets = c.take<int32_t>((size_t)(experts + 1) * 4);
  p.active = c.take<int32_t>((size_t)experts * 4);
  p.active_count = c.take<int32_t>(4);
  p.sws_bytes = sort_workspace_bytes(n, experts);
  p.sws = c.take<char>(p.sws_bytes);
  p.h = c.take<char>((size_t)n * intermediate * act_bytes(act));
  p.x16 = c.take<char>((size_t)n * hidden * 2);  // slot-ordered f16 operand
  p.h16 = c.take<char>((size_t)n * intermediate * 2);
  p.used = c.used;
  return p;
}

int tf_moe_expert_workspace_size(int64_t n, int64_t x_rows, int32_t hidden, int32_t intermediate,
                                 int32_t experts, int act, size_t* bytes) {
  if (!bytes || n < 0 || x_rows < 0 || hidden <= 0 || intermediate <= 0 || experts <= 0)
    return set_error(TF_ERR_INVALID_ARGUMENT, "bad arguments");
  TF_TRY(check_act(act));
  *bytes = plan_expert(nullptr, 0, n, x_rows, hidden, intermediate, experts, act).used;
  return TF_OK;
}

// ordered: out rows in the routes' own order (the down projection writes
// slot n's row to order[n]); inverse then lives in the workspace.
static tf_status expert_gpu(const void* x, int64_t x_rows, int32_t hidden, const int32_t* token_indices,
                            const int32_t* expert_ids, int64_t n, int32_t intermediate, int32_t experts,
                            const tf_affine_weight* gate, const tf_affine_weight* up,
                            const tf_affine_weight* down, int act, void* out, int32_t* inverse, bool ordered,
                            void* workspace, size_t workspace_bytes, void* stream) {
  TF_TRY(check_act(act));
  if (n < 0 || n > INT32_MAX || x_rows < 0 || hidden <= 0 || hidden % 64 || experts <= 0 || experts > 256)
    return set_error(TF_ERR_SHAPE, "expert hook route arrays must be parallel integer vectors");
  TF_TRY(check_affine(gate, "gate_proj", true));
  TF_TRY(check_affine(up, "up_proj", true));
  TF_TRY(check_affine(down, "down_proj", true));
  if (gate->in_features != hidden || up->in_features != hidden || down->out_features != hidden ||
      gate->out_features != intermediate || up->out_features != intermediate ||
      down->in_features != intermediate || gate->experts != experts || up->experts != experts ||
      down->experts != experts)
    return set_error(TF_ERR_SHAPE, "expert hook: packed parameter geometry differs");
  if (workspace_bytes < plan_expert(nullptr, 0, n, x_rows, hidden, intermediate, experts, act).used)
    return set_error(TF_ERR_INVALID_ARGUMENT, "expert hook: workspace too small");
  if (n == 0) return TF_OK;
  if (!x || !token_indices || !expert_ids || !out || (!inverse && !ordered) || !workspace || !aligned16(x))
    return set_error(TF_ERR_INVALID_ARGUMENT, "expert hook: NULL or unaligned pointer");
  cudaStream_t s = st(stream);
  const ExpertPlan w = plan_expert(workspace, workspace_bytes, n, x_rows, hidden, intermediate, experts, act);
  if (ordered) inverse = w.inverse;
  int32_t* order = w.order;
  int32_t* xrow = w.xrow;
  int32_t* offsets = w.offsets;
  int32_t* active = w.active;
  int32_t* active_count = w.active_count;
  void* h = w.h;
  TF_TRY(launch_route_sort(expert_ids, n, experts, order, inverse, offsets, active, active_count, w.sws,
                           w.sws_bytes, s));
  TF_TRY(launch_gather_index(token_indices, order, n, 1, xrow, s));
  QmmProblem p;
  p.mode = QMM_GROUPED;
  p.epilogue = EPI_SWIGLU;
  p.act = act;
  p.x = x;
  p.x_stride = hidden;
  p.x_index = xrow;
  p.n = n;
  p.offsets = offsets;
  p.active = active;
  p.active_count = active_count;
  p.w0 = *gate;
  p.w1 = *up;
  p.y = h;
  p.y_stride = intermediate;
  QmmProblem d = p;
  d.epilogue = EPI_PLAIN;
  d.x = h;
  d.x_stride = intermediate;
  d.x_index = nullptr;
  d.w0 = *down;
  d.y = out;
  d.y_stride = hidden;
  d.y_index = ordered ? order : nullptr;
  const bool tc_up = qmm_uses_tc(p), tc_dn = qmm_uses_tc(d);
  if (tc_up) {
    TF_TRY(launch_gather_f16(x, hidden, act, xrow, 1, n, hidden, w.x16, 1, s));
    p.x16 = w.x16;
    p.x16_perm = 1;
    if (tc_dn) {
      p.y_f16 = 1;
      d.x16 = h;
      d.x16_perm = 1;
    }
  }
  TF_TRY(launch_qmm(p, s));
  if (tc_dn && !p.y_f16) {
    TF_TRY(launch_gather_f16(h, intermediate, act, nullptr, 1, n, intermediate, w.h16, 1, s));
    d.x16 = w.h16;
    d.x16_perm = 1;
  }
  return launch_qmm(d, s);
}

int tf_moe_expert_gpu(const void* x, int64_t x_rows, int32_t hidden, const int32_t* token_indices,
                      const int32_t* expert_ids, int64_t n, int experts_sorted, int32_t intermediate,
                      int32_t experts, const tf_affine_weight* gate, const tf_affine_weight* up,
                      const tf_affine_weight* down, int act, void* out_sorted, int32_t* inverse,
                      void* workspace, size_t workspace_bytes, void* stream) {
  (void)experts_sorted;  // the stable sort of sorted ids is the identity
  return expert_gpu(x, x_rows, hidden, token_indices, expert_ids, n, intermediate, experts, gate, up, down, act,
                    out_sorted, inverse, false, workspace, workspace_bytes, stream);
}

int tf_moe_expert_gpu_ordered(const void* x, int64_t x_rows, int32_t hidden, const int32_t* token_indices,
                              const int32_t* expert_ids, int64_t n, int32_t intermediate, int32_t experts,
                              const tf_affine_weight* gate, const tf_affine_weight* up,
                              const tf_affine_weight* down, int act, void* out, void* workspace,
                              size_t workspace_bytes, void* stream) {
  return expert_gpu(x, x_rows, hidden, token_indices, expert_ids, n, intermediate, experts, gate, up, down, act,
                    out, nullptr, true, workspace, workspace_bytes, stream);
}

int tf_gather_rows(const void* x, int64_t x_rows, int32_t width, const int32_t* index, int32_t div, int64_t n,
                   int act, void* y, void* stream) {
  TF_TRY(check_act(act));
  if (n < 0 || x_rows < 0 || width <= 0 || width % 8 || div <= 0)
    return set_error(TF_ERR_SHAPE, "gather_rows: bad geometry");
  if (n == 0) return TF_OK;
  if (!x || !index || !y || !aligned16(x) || !aligned16(y))
    return set_error(TF_ERR_INVALID_ARGUMENT, "gather_rows: NULL or unaligned pointer");
  return launch_gather_rows(x, width, index, div, n, width, act, y, st(stream));
}

// ---------------------------------------------------------------- attention

int tf_attention_decode_workspace_size(int32_t batch, int32_t heads, int32_t capacity, size_t* bytes) {
  if (!bytes || batch < 0 || heads <= 0 || capacity <= 0)
    return set_error(TF_ERR_INVALID_ARGUMENT, "bad arguments");
  *bytes = attention_ws_bytes(batch, heads, capacity, TF_DTYPE_F16);
  return TF_OK;
}

int tf_attention_decode(const void* qkv, int32_t batch, int32_t heads, int32_t head_dim,
                        const void* q_norm, const void* k_norm, float eps, float rope_theta,
                        const int32_t* positions, int32_t max_length, void* k_cache, void* v_cache,
                        int32_t capacity, float scale, int act, void* out, void* workspace,
                        size_t workspace_bytes, void* stream) {
  TF_TRY(check_act(act));
  if (batch < 0 || heads <= 0 || head_dim <= 0 || capacity <= 0)
    return set_error(TF_ERR_SHAPE, "attention: bad geometry");
  if (max_length < 1 || max_length > capacity)
    return set_error(TF_ERR_CAPACITY, "attention: max_length %d outside [1, capacity %d]", max_length,
                     capacity);
  if (!(eps > 0) || !(rope_theta > 1) || !(scale > 0))
    return set_error(TF_ERR_INVALID_ARGUMENT, "attention: eps, theta and scale must be positive");
  if (batch == 0) return TF_OK;
  if (!qkv || !q_norm || !k_norm || !positions || !k_cache || !v_cache || !out || !workspace ||
      !aligned16(qkv) || !aligned16(k_cache) || !aligned16(v_cache))
    return set_error(TF_ERR_INVALID_ARGUMENT, "attention: NULL or unaligned pointer");
  AttnProblem a;
  a.qkv = qkv;
  a.rows = batch;
  a.heads = heads;
  a.head_dim = head_dim;
  a.q_norm = q_norm;
  a.k_norm = k_norm;
  a.eps = eps;
  a.theta = rope_theta;
  a.pos = positions;
  a.req = nullptr;
  a.max_len = max_length;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.capacity = capacity;
  a.scale = scale;
  a.act = act;
  a.out = out;
  a.ws = workspace;
  a.ws_bytes = workspace_bytes;
  return launch_attention(a, st(stream));
}

}  // extern "C"
