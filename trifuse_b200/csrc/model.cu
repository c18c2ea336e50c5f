// Device-resident OLMoE model and the per-request session (KV cache +
// scratch) driving the decode / prefill forward.
//
// Restates NativeGraniteMoEPrefill (MLXNativeGraniteMoEPrefill.h:155-493) for
// architecture OLMoE: the constructor's name binding and geometry checks
// (157-330) become tf_model_create / tf_model_bind / tf_model_finalize, and
// run() (347-493) becomes forward_rows(): embedding -> L x (input RMSNorm,
// fused q|k|v QMM, attention, o-proj + residual, post RMSNorm, MoE block) ->
// final RMSNorm of each request's last row -> lm_head (fp32 logits).
//
// Layout in HBM: all weights live in one arena.  The q, k and v projections
// of a layer are stored back to back as one [3W][H] packed matrix so the three
// projections are one launch.  KV caches are f16
// [max_batch][kv_heads][capacity][head_dim] per layer (BHSD, as the
// reference's Pool, patches/executorch.patch:1834-2094).
#include <atomic>
#include <map>
#include <string>
#include <cmath>
#include <tuple>
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "internal.h"

using namespace tf;

namespace {

struct Role {
  char* ptr = nullptr;
  size_t bytes = 0;
  bool bound = false;
};

struct LayerW {
  const __half* input_norm;
  const __half* post_norm;
  const __half* q_norm;
  const __half* k_norm;
  tf_affine_weight qkv;
  tf_affine_weight o;
  tf_affine_weight router;
  tf_affine_weight gate, up, down;
};

tf_affine_weight affine(char* q, char* s, char* b, int experts, int out, int in) {
  tf_affine_weight w;
  w.q = reinterpret_cast<const uint32_t*>(q);
  w.scales = s;
  w.biases = b;
  w.experts = experts;
  w.out_features = out;
  w.in_features = in;
  w.group_size = 64;
  w.bits = 4;
  return w;
}

}  // namespace

struct tf_model {
  tf_olmoe_config c{};
  int device = 0;
  char* arena = nullptr;
  size_t arena_bytes = 0;
  std::map<std::string, Role> roles;
  tf_affine_weight embed{}, lm_head{};
  const __half* final_norm = nullptr;
  std::vector<LayerW> layers;
  bool finalized = false;
  int sessions = 0;
};

namespace {

// Event-pair recorder behind tf_session_trace.
struct SessionTracer : Tracer {
  struct Pair {
    int phase;
    cudaEvent_t a, b;
  };
  std::vector<cudaEvent_t> pool;
  std::vector<Pair> pairs;
  int open_phase = -1;
  cudaEvent_t open_ev = nullptr;
  cudaEvent_t get() {
    if (!pool.empty()) {
      cudaEvent_t e = pool.back();
      pool.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }
  void mark(int phase, bool begin, cudaStream_t s) override {
    if (begin) {
      open_phase = phase;
      open_ev = get();
      cudaEventRecord(open_ev, s);
    } else if (open_phase == phase) {
      cudaEvent_t e = get();
      cudaEventRecord(e, s);
      pairs.push_back({phase, open_ev, e});
      open_phase = -1;
    }
  }
  void recycle() {
    for (auto& p : pairs) {
      pool.push_back(p.a);
      pool.push_back(p.b);
    }
    pairs.clear();
  }
  ~SessionTracer() override {
    recycle();
    for (auto e : pool) cudaEventDestroy(e);
  }
};

struct TraceScope {
  explicit TraceScope(Tracer* t) { g_tracer = t; }
  ~TraceScope() { g_tracer = nullptr; }
};

}  // namespace

struct tf_session {
  tf_model* m = nullptr;
  int max_batch = 0;
  int capacity = 0;
  int max_rows = 0;
  char* kv = nullptr;
  std::vector<void*> k, v;
  std::vector<int32_t> lengths;
  char* scratch = nullptr;
  void* h0 = nullptr;
  void* h1 = nullptr;
  void* xn = nullptr;
  void* qkv = nullptr;
  void* attn = nullptr;
  void* x16 = nullptr;  // f16 operand copy (bf16 models, tensor-core projections)
  void* hc = nullptr;   // [max_batch][H] residual rows of the last layer's queries (prefill)
  int64_t* ids = nullptr;
  int32_t* pos = nullptr;
  int32_t* req = nullptr;
  int32_t* last_rows = nullptr;
  float* logits = nullptr;  // [max_batch][vocab]
  int64_t* greedy = nullptr;  // [max_batch] greedy tokens before a host copy
  int4* qblocks = nullptr;    // prefill query blocks {row, rows, request, position}
  void* attn_ws = nullptr;
  void* rope = nullptr;  // float2 [capacity][head_dim / 2] RoPE (cos, sin)
  size_t attn_ws_bytes = 0;
  void* moe_ws = nullptr;
  size_t moe_ws_bytes = 0;
  // Split-schedule buffers of the dense tensor-core projections (the MoE
  // block carries its own inside moe_ws); counters zeroed at creation and
  // on reset, left zero by every completed launch.
  float* split_partials = nullptr;
  int* split_counters = nullptr;
  std::atomic<int> cancelled{0};
  // Set by a failure after work was dispatched (a launch or CUDA error, a
  // cancellation between layers, or a device-side error found at a
  // completion point); every call but reset is refused while it is set.
  bool invalid = false;
  bool tracing = false;
  // Diagnostic capture (tf_session_capture): each layer's top-k expert ids
  // and output hidden states of a forward land at route_capture + layer *
  // rows * k and hidden_capture + layer * rows * hidden.
  int32_t* route_capture = nullptr;
  void* hidden_capture = nullptr;
  int64_t capture_rows = 0;
  SessionTracer tracer;
  // Decode steps as CUDA graphs, one per (batch, with logits, attention
  // splits of 256 keys, QMM path): the first step of a shape runs eagerly,
  // the second is captured on gstream, later ones replay it.
  struct DecodeGraph {
    cudaGraphExec_t exec = nullptr;
    int64_t launches = 0;
    int eager_runs = 0;
  };
  bool graphs_on = true;
  cudaStream_t gstream = nullptr;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  std::map<std::tuple<int, int, int, int>, DecodeGraph> graphs;
};

namespace {

// Scoped device switch.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int d) {
    cudaGetDevice(&prev);
    if (prev != d) cudaSetDevice(d);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

tf_status validate_config(const tf_olmoe_config* c) {
  // NativeGraniteMoEPrefill::validate_config (MLXNativeGraniteMoEPrefill.h:306-330).
  if (!c) return set_error(TF_ERR_INVALID_ARGUMENT, "config is NULL");
  const int32_t vals[] = {c->layers, c->hidden, c->heads, c->kv_heads, c->head_dim, c->intermediate,
                          c->vocab, c->experts, c->top_k, c->capacity};
  for (int32_t v : vals)
    if (v <= 0) return set_error(TF_ERR_SHAPE, "invalid model geometry");
  if (c->heads % c->kv_heads || c->head_dim % 2 || (int64_t)c->heads * c->head_dim != c->hidden ||
      c->top_k > c->experts || c->hidden % 64 || c->intermediate % 64 ||
      (int64_t)c->capacity * c->top_k > INT32_MAX)
    return set_error(TF_ERR_SHAPE, "unsupported attention/expert geometry");
  if (!(c->rms_eps > 0) || !(c->rope_theta > 1))
    return set_error(TF_ERR_INVALID_ARGUMENT, "invalid normalization/RoPE configuration");
  if (c->kv_heads != c->heads)
    return set_error(TF_ERR_UNSUPPORTED, "grouped-query attention is not on this path (kv_heads %d != heads %d)",
                     c->kv_heads, c->heads);
  if (c->head_dim != 128) return set_error(TF_ERR_UNSUPPORTED, "head_dim %d (only 128)", c->head_dim);
  if (c->hidden % 256 || c->hidden > 2048) return set_error(TF_ERR_UNSUPPORTED, "hidden %d (router supports <= 2048)", c->hidden);
  if (c->experts > 64 || c->top_k > 32) return set_error(TF_ERR_UNSUPPORTED, "experts <= 64, top_k <= 32");
  if (!act_ok(c->act)) return set_error(TF_ERR_INVALID_ARGUMENT, "activation dtype must be f16 or bf16");
  return TF_OK;
}

// Device-side failures recorded since the last check, as a status: an
// expired tensor-core pipeline wait (codes 11-51), an activation beyond the
// f16 range reaching a tensor-core operand (5), a token id past the
// embedding table (6).  Clears the flags.  The stream has been synchronized.
tf_status device_status() {
  const int tc = read_tc_error(true);
  const int emb = read_embed_error(true);
  if (tc >= 11)
    return set_error(TF_ERR_TIMEOUT, "a tensor-core pipeline wait expired (device code %d); results are incomplete", tc);
  if (tc == 5)
    return set_error(TF_ERR_STATE, "an activation beyond the f16 range reached a tensor-core operand (device code 5)");
  if (tc) return set_error(TF_ERR_STATE, "device error code %d", tc);
  if (emb == 6) return set_error(TF_ERR_STATE, "a token id past the embedding table was read as row 0 (device code 6)");
  return TF_OK;
}

// A failure after dispatch invalidates the session until tf_session_reset,
// after the submitted work drained (TFETResidentSession.mm:388-392 quarantine,
// failDispatched at :667; patches/executorch.patch:1486-1499 maps the error).
tf_status invalidate(tf_session* s, tf_status rc, cudaStream_t st) {
  s->invalid = true;
  cudaStreamSynchronize(st);
  if (s->gstream) cudaStreamSynchronize(s->gstream);
  return rc;
}

tf_status refuse_invalid(const tf_session* s) {
  return set_error(TF_ERR_STATE, "Resident session is invalid after a dispatched failure; tf_session_reset re-admits it");
}

}  // namespace

extern "C" {

int tf_model_create(const tf_olmoe_config* config, int device, tf_model** model) {
  if (!model) return set_error(TF_ERR_INVALID_ARGUMENT, "model out-pointer is NULL");
  *model = nullptr;
  TF_TRY(validate_config(config));
  const tf_olmoe_config& c = *config;
  auto* m = new tf_model();
  m->c = c;
  m->device = device;
  const int H = c.hidden, W = c.heads * c.head_dim, Wkv = c.kv_heads * c.head_dim, E = c.experts,
            I = c.intermediate, V = c.vocab;
  // Role table: (name, bytes) in arena order.  q/k/v parts of one layer are
  // adjacent so that they form one [W + 2 Wkv][H] packed matrix.
  std::vector<std::pair<std::string, size_t>> order;
  auto add_affine = [&](const std::string& name, int64_t rows, int64_t in) {
    order.push_back({name + ".weight", (size_t)rows * in / 2});
  };
  auto add_sb = [&](const std::string& name, int64_t rows, int64_t in) {
    order.push_back({name + ".scales", (size_t)rows * (in / 64) * 2});
    order.push_back({name + ".biases", (size_t)rows * (in / 64) * 2});
  };
  add_affine("model.embed_tokens", V, H);
  add_sb("model.embed_tokens", V, H);
  add_affine("lm_head", V, H);
  add_sb("lm_head", V, H);
  order.push_back({"model.norm.weight", (size_t)H * 2});
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    order.push_back({p + "input_layernorm.weight", (size_t)H * 2});
    order.push_back({p + "post_attention_layernorm.weight", (size_t)H * 2});
    order.push_back({p + "self_attn.q_norm.weight", (size_t)W * 2});
    order.push_back({p + "self_attn.k_norm.weight", (size_t)Wkv * 2});
    add_affine(p + "self_attn.q_proj", W, H);
    add_affine(p + "self_attn.k_proj", Wkv, H);
    add_affine(p + "self_attn.v_proj", Wkv, H);
    order.push_back({p + "self_attn.q_proj.scales", (size_t)W * (H / 64) * 2});
    order.push_back({p + "self_attn.k_proj.scales", (size_t)Wkv * (H / 64) * 2});
    order.push_back({p + "self_attn.v_proj.scales", (size_t)Wkv * (H / 64) * 2});
    order.push_back({p + "self_attn.q_proj.biases", (size_t)W * (H / 64) * 2});
    order.push_back({p + "self_attn.k_proj.biases", (size_t)Wkv * (H / 64) * 2});
    order.push_back({p + "self_attn.v_proj.biases", (size_t)Wkv * (H / 64) * 2});
    add_affine(p + "self_attn.o_proj", H, W);
    add_sb(p + "self_attn.o_proj", H, W);
    add_affine(p + "mlp.gate", E, H);
    add_sb(p + "mlp.gate", E, H);
    for (const char* n : {"gate_proj", "up_proj"}) {
      add_affine(p + "mlp.switch_mlp." + n, (int64_t)E * I, H);
      add_sb(p + "mlp.switch_mlp." + n, (int64_t)E * I, H);
    }
    add_affine(p + "mlp.switch_mlp.down_proj", (int64_t)E * H, I);
    add_sb(p + "mlp.switch_mlp.down_proj", (int64_t)E * H, I);
  }
  // q|k|v parts must be contiguous: no padding between them.
  size_t total = 0;
  std::vector<size_t> offs;
  for (size_t i = 0; i < order.size(); ++i) {
    const std::string& n = order[i].first;
    const bool packed_part = n.find("self_attn.k_proj") != std::string::npos ||
                             n.find("self_attn.v_proj") != std::string::npos;
    if (!packed_part) total = align_up(total, 256);
    offs.push_back(total);
    total += order[i].second;
  }
  total = align_up(total, 256);
  {
    DeviceGuard g(device);
    const cudaError_t e = cudaMalloc(&m->arena, total);
    if (e != cudaSuccess) {
      delete m;
      return set_error(TF_ERR_OUT_OF_MEMORY, "model arena of %zu bytes: %s", total, cudaGetErrorString(e));
    }
  }
  m->arena_bytes = total;
  for (size_t i = 0; i < order.size(); ++i) m->roles[order[i].first] = Role{m->arena + offs[i], order[i].second, false};
  auto R = [&](const std::string& n) { return m->roles.at(n).ptr; };
  m->embed = affine(R("model.embed_tokens.weight"), R("model.embed_tokens.scales"),
                    R("model.embed_tokens.biases"), 0, V, H);
  m->lm_head = affine(R("lm_head.weight"), R("lm_head.scales"), R("lm_head.biases"), 0, V, H);
  m->final_norm = (const __half*)R("model.norm.weight");
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    LayerW L;
    L.input_norm = (const __half*)R(p + "input_layernorm.weight");
    L.post_norm = (const __half*)R(p + "post_attention_layernorm.weight");
    L.q_norm = (const __half*)R(p + "self_attn.q_norm.weight");
    L.k_norm = (const __half*)R(p + "self_attn.k_norm.weight");
    L.qkv = affine(R(p + "self_attn.q_proj.weight"), R(p + "self_attn.q_proj.scales"),
                   R(p + "self_attn.q_proj.biases"), 0, W + 2 * Wkv, H);
    L.o = affine(R(p + "self_attn.o_proj.weight"), R(p + "self_attn.o_proj.scales"),
                 R(p + "self_attn.o_proj.biases"), 0, H, W);
    L.router = affine(R(p + "mlp.gate.weight"), R(p + "mlp.gate.scales"), R(p + "mlp.gate.biases"), 0, E, H);
    const std::string s = p + "mlp.switch_mlp.";
    L.gate = affine(R(s + "gate_proj.weight"), R(s + "gate_proj.scales"), R(s + "gate_proj.biases"), E, I, H);
    L.up = affine(R(s + "up_proj.weight"), R(s + "up_proj.scales"), R(s + "up_proj.biases"), E, I, H);
    L.down = affine(R(s + "down_proj.weight"), R(s + "down_proj.scales"), R(s + "down_proj.biases"), E, H, I);
    m->layers.push_back(L);
  }
  *model = m;
  return TF_OK;
}

int tf_model_bind(tf_model* model, const char* name, const void* data, size_t bytes, int data_on_device) {
  if (!model || !name || !data) return set_error(TF_ERR_INVALID_ARGUMENT, "bind: NULL argument");
  if (model->finalized) return set_error(TF_ERR_STATE, "bind: model already finalized");
  auto it = model->roles.find(name);
  if (it == model->roles.end())
    return set_error(TF_ERR_INVALID_ARGUMENT, "unexpected constant/unsupported model structure: %s", name);
  Role& r = it->second;
  if (r.bound) return set_error(TF_ERR_STATE, "missing/aliased parameter role: %s bound twice", name);
  if (bytes != r.bytes)
    return set_error(TF_ERR_SHAPE, "packed parameter geometry differs: %s has %zu bytes, expected %zu", name,
                     bytes, r.bytes);
  DeviceGuard g(model->device);
  TF_CUDA(cudaMemcpy(r.ptr, data, bytes, data_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
  // A device-to-device cudaMemcpy may return before the copy ran; the caller
  // may reuse the source as soon as this returns.
  if (data_on_device) TF_CUDA(cudaDeviceSynchronize());
  r.bound = true;
  return TF_OK;
}

int tf_model_finalize(tf_model* model) {
  if (!model) return set_error(TF_ERR_INVALID_ARGUMENT, "model is NULL");
  for (const auto& kv : model->roles)
    if (!kv.second.bound) return set_error(TF_ERR_STATE, "missing parameter role: %s", kv.first.c_str());
  model->finalized = true;
  return TF_OK;
}

int tf_model_destroy(tf_model* model) {
  if (!model) return TF_OK;
  if (model->sessions > 0) return set_error(TF_ERR_STATE, "model still has %d sessions", model->sessions);
  DeviceGuard g(model->device);
  cudaFree(model->arena);
  delete model;
  return TF_OK;
}

int tf_session_create(tf_model* model, int32_t max_batch, int32_t capacity, int32_t max_prefill_tokens,
                      tf_session** session) {
  if (!session) return set_error(TF_ERR_INVALID_ARGUMENT, "session out-pointer is NULL");
  *session = nullptr;
  if (!model || !model->finalized) return set_error(TF_ERR_STATE, "model missing or not finalized");
  if (max_batch <= 0 || capacity <= 0 || max_prefill_tokens < 0)
    return set_error(TF_ERR_INVALID_ARGUMENT, "session: bad sizes");
  const tf_olmoe_config& c = model->c;
  if (capacity > c.capacity)
    return set_error(TF_ERR_CAPACITY, "Runtime capacity %d must not extend the model's %d", capacity, c.capacity);
  auto* s = new tf_session();
  s->m = model;
  s->max_batch = max_batch;
  s->capacity = capacity;
  s->max_rows = max_batch > max_prefill_tokens ? max_batch : max_prefill_tokens;
  s->lengths.assign(max_batch, 0);
  const int H = c.hidden, W = c.heads * c.head_dim, Wkv = c.kv_heads * c.head_dim;
  const int64_t R = s->max_rows;
  const size_t per_cache = (size_t)max_batch * c.kv_heads * capacity * c.head_dim * 2;
  tf_moe_args ma{};
  ma.tokens = R;
  ma.hidden = H;
  ma.intermediate = c.intermediate;
  ma.experts = c.experts;
  ma.top_k = c.top_k;
  ma.act = c.act;
  s->moe_ws_bytes = moe_workspace_bytes(&ma);
  s->attn_ws_bytes = attention_ws_bytes(R, c.heads, capacity, c.act);
  Carve cv(nullptr, 0);
  auto plan = [&](Carve& k) {
    s->h0 = k.take<char>((size_t)R * H * 2);
    s->h1 = k.take<char>((size_t)R * H * 2);
    s->xn = k.take<char>((size_t)R * H * 2);
    s->qkv = k.take<char>((size_t)R * (W + 2 * Wkv) * 2);
    s->attn = k.take<char>((size_t)R * W * 2);
    s->x16 = k.take<char>((size_t)R * (H > W ? H : W) * 2);
    s->hc = k.take<char>((size_t)max_batch * H * 2);
    s->ids = k.take<int64_t>((size_t)R * 8);
    s->pos = k.take<int32_t>((size_t)R * 4);
    s->req = k.take<int32_t>((size_t)R * 4);
    s->last_rows = k.take<int32_t>((size_t)max_batch * 4);
    s->logits = k.take<float>((size_t)max_batch * c.vocab * 4);
    s->greedy = k.take<int64_t>((size_t)max_batch * 8);
    s->qblocks = k.take<int4>((size_t)(R / kPrefillQueryBlock + max_batch + 1) * sizeof(int4));
    s->attn_ws = k.take<char>(s->attn_ws_bytes);
    s->rope = k.take<float>((size_t)capacity * (c.head_dim / 2) * 8);
    s->moe_ws = k.take<char>(s->moe_ws_bytes);
    s->split_partials = k.take<float>(qmm_split_partial_bytes());
    s->split_counters = k.take<int>((size_t)kQmmSplitCounters * sizeof(int));
  };
  plan(cv);
  DeviceGuard g(model->device);
  cudaError_t e = cudaMalloc(&s->kv, per_cache * 2 * c.layers);
  if (e != cudaSuccess) {
    delete s;
    return set_error(TF_ERR_OUT_OF_MEMORY, "KV cache of %zu bytes: %s", per_cache * 2 * c.layers,
                     cudaGetErrorString(e));
  }
  e = cudaMalloc(&s->scratch, cv.used);
  if (e != cudaSuccess) {
    cudaFree(s->kv);
    delete s;
    return set_error(TF_ERR_OUT_OF_MEMORY, "session scratch of %zu bytes: %s", cv.used, cudaGetErrorString(e));
  }
  Carve real(s->scratch, cv.used);
  plan(real);
  // The split counters (in moe_ws and split_counters) start at zero.
  e = cudaMemset(s->scratch, 0, cv.used);
  if (e != cudaSuccess) {
    cudaFree(s->kv);
    cudaFree(s->scratch);
    delete s;
    return set_error(TF_ERR_CUDA, "session scratch clear: %s", cudaGetErrorString(e));
  }
  if (c.head_dim == 128) {
    const tf_status rs = launch_rope_table(c.rope_theta, capacity, s->rope, 0);
    if (rs == TF_OK) e = cudaStreamSynchronize(0);
    if (rs != TF_OK || e != cudaSuccess) {
      cudaFree(s->kv);
      cudaFree(s->scratch);
      delete s;
      return rs != TF_OK ? rs : set_error(TF_ERR_CUDA, "RoPE table: %s", cudaGetErrorString(e));
    }
  } else {
    s->rope = nullptr;
  }
  for (int l = 0; l < c.layers; ++l) {
    s->k.push_back(s->kv + per_cache * (2 * l));
    s->v.push_back(s->kv + per_cache * (2 * l + 1));
  }
  if (cudaStreamCreateWithFlags(&s->gstream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&s->ev_in, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&s->ev_out, cudaEventDisableTiming) != cudaSuccess)
    s->graphs_on = false;  // decode then always runs eagerly
  model->sessions++;
  *session = s;
  return TF_OK;
}

int tf_session_destroy(tf_session* s) {
  if (!s) return TF_OK;
  DeviceGuard g(s->m->device);
  for (auto& kv : s->graphs)
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
  if (s->ev_in) cudaEventDestroy(s->ev_in);
  if (s->ev_out) cudaEventDestroy(s->ev_out);
  if (s->gstream) cudaStreamDestroy(s->gstream);
  cudaFree(s->kv);
  cudaFree(s->scratch);
  s->m->sessions--;
  delete s;
  return TF_OK;
}

int tf_session_kv(tf_session* s, int32_t layer, void** k_cache, void** v_cache) {
  if (!s || !k_cache || !v_cache) return set_error(TF_ERR_INVALID_ARGUMENT, "NULL argument");
  if (layer < 0 || layer >= s->m->c.layers) return set_error(TF_ERR_INVALID_ARGUMENT, "layer out of range");
  *k_cache = s->k[layer];
  *v_cache = s->v[layer];
  return TF_OK;
}

int tf_session_set_lengths(tf_session* s, const int32_t* lengths, int32_t batch) {
  if (!s || (!lengths && batch)) return set_error(TF_ERR_INVALID_ARGUMENT, "NULL argument");
  if (batch < 0 || batch > s->max_batch) return set_error(TF_ERR_INVALID_ARGUMENT, "batch out of range");
  for (int b = 0; b < batch; ++b)
    if (lengths[b] < 0 || lengths[b] > s->capacity)
      return set_error(TF_ERR_CAPACITY, "length %d of request %d outside [0, %d]", lengths[b], b, s->capacity);
  for (int b = 0; b < batch; ++b) s->lengths[b] = lengths[b];
  return TF_OK;
}

int tf_session_get_lengths(tf_session* s, int32_t* lengths, int32_t batch) {
  if (!s || (!lengths && batch)) return set_error(TF_ERR_INVALID_ARGUMENT, "NULL argument");
  if (batch < 0 || batch > s->max_batch) return set_error(TF_ERR_INVALID_ARGUMENT, "batch out of range");
  for (int b = 0; b < batch; ++b) lengths[b] = s->lengths[b];
  return TF_OK;
}

int tf_session_cancel(tf_session* s) {
  if (!s) return set_error(TF_ERR_INVALID_ARGUMENT, "session is NULL");
  s->cancelled.store(1);
  return TF_OK;
}

int tf_session_reset(tf_session* s) {
  if (!s) return set_error(TF_ERR_INVALID_ARGUMENT, "session is NULL");
  DeviceGuard g(s->m->device);
  if (s->invalid) {
    // After a dispatched failure: wait for the device, clear its error flags
    // and the arrival counters a stopped launch may have left behind (split
    // tiles and route sort in the MoE workspace, split attention).
    TF_CUDA(cudaDeviceSynchronize());
    read_tc_error(true);
    read_embed_error(true);
    TF_CUDA(cudaMemset(s->moe_ws, 0, s->moe_ws_bytes));
    TF_CUDA(cudaMemset(s->attn_ws, 0, s->attn_ws_bytes));
    TF_CUDA(cudaMemset(s->split_counters, 0, (size_t)kQmmSplitCounters * sizeof(int)));
    s->invalid = false;
  }
  s->cancelled.store(0);
  for (auto& l : s->lengths) l = 0;
  return TF_OK;
}

int tf_session_check(tf_session* s, void* stream) {
  if (!s) return set_error(TF_ERR_INVALID_ARGUMENT, "session is NULL");
  if (s->invalid) return refuse_invalid(s);
  DeviceGuard g(s->m->device);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return invalidate(s, set_error(TF_ERR_CUDA, "session check: %s", cudaGetErrorString(e)), st);
  const tf_status rc = device_status();
  return rc == TF_OK ? TF_OK : invalidate(s, rc, st);
}

}  // extern "C"

namespace {

// Dense projection; with bf16 activations on the tensor-core path the input
// rows are first copied to f16 (the MMA operand dtype) in the tensor-core
// operand order.  f16 activations are read in place.
tf_status dense_qmm(tf_session* s, QmmProblem& q, int64_t x_rows, cudaStream_t st) {
  q.partials = s->split_partials;
  q.partial_bytes = qmm_split_partial_bytes();
  q.counters = s->split_counters;
  q.counter_cap = kQmmSplitCounters;
  if (q.act == TF_DTYPE_BF16 && qmm_uses_tc(q)) {
    TF_TRY(launch_bf16_to_f16(q.x, x_rows * q.x_stride, s->x16, 1, st));
    q.x16 = s->x16;
    q.x16_perm = 1;
  }
  return launch_qmm(q, st);
}

// Forward `rows` token rows through every layer.  Inputs already on device:
// s->ids [rows], s->pos [rows], s->req [rows] (or identity when req_ident).
// Leaves the final hidden states in s->h0.
//
// Prefill (`last` = the nlast device rows that end a request, fewer than
// `rows`): as the reference, the last layer appends K/V of every row but
// runs attention, o-proj and the MoE block only for those rows
// (MLXNativeGraniteMoEPrefill.h:440-442, 471), leaving their hidden states
// compact in s->h0 rows 0..nlast-1; a cache-only call (`cache_only`) stops
// after that layer's K/V write (:470).
tf_status forward_rows(tf_session* s, int64_t rows, bool req_ident, int max_len, cudaStream_t st,
                       int nqblocks = 0, const int32_t* last = nullptr, int nlast = 0, bool cache_only = false) {
  const tf_model* m = s->m;
  const tf_olmoe_config& c = m->c;
  const int H = c.hidden, W = c.heads * c.head_dim;
  const int QKV = W + 2 * c.kv_heads * c.head_dim;
  trace(PH_EMBED, true, st);
  TF_TRY(launch_embedding(s->ids, rows, m->embed, c.act, s->h0, st));
  trace(PH_EMBED, false, st);
  bool normed = false;  // s->xn already holds this layer's input norm (fused into the previous combine)
  for (int l = 0; l < c.layers; ++l) {
    if (s->cancelled.load()) return set_error(TF_ERR_CANCELLED, "cancelled before layer %d", l);
    const LayerW& L = m->layers[l];
    // Last layer of a prefill: queries of the requests' last rows only.
    const bool lq = last && nlast < rows && l == c.layers - 1;
    if (!normed) {
      trace(PH_INPUT_NORM, true, st);
      TF_TRY(launch_rms_norm(s->h0, rows, H, L.input_norm, c.rms_eps, c.act, s->xn, st));
      trace(PH_INPUT_NORM, false, st);
    }
    normed = false;
    QmmProblem q;
    q.mode = QMM_DENSE;
    q.act = c.act;
    q.x = s->xn;
    q.x_stride = H;
    q.n = rows;
    q.w0 = L.qkv;
    q.y = s->qkv;
    q.y_stride = QKV;
    trace(PH_QKV, true, st);
    TF_TRY(dense_qmm(s, q, rows, st));
    trace(PH_QKV, false, st);
    AttnProblem a;
    a.qkv = s->qkv;
    a.rows = rows;
    a.heads = c.heads;
    a.head_dim = c.head_dim;
    a.q_norm = L.q_norm;
    a.k_norm = L.k_norm;
    a.eps = c.rms_eps;
    a.theta = c.rope_theta;
    a.rope = s->rope;
    a.arrivals_zero = true;
    a.ws_rows = s->max_rows;
    a.pos = s->pos;
    a.req = req_ident ? nullptr : s->req;
    a.max_len = max_len;
    a.k_cache = s->k[l];
    a.v_cache = s->v[l];
    a.capacity = s->capacity;
    a.scale = (float)(1.0 / sqrt((double)c.head_dim));
    a.act = c.act;
    a.out = s->attn;
    a.ws = s->attn_ws;
    a.ws_bytes = s->attn_ws_bytes;
    a.qblocks = nqblocks ? s->qblocks : nullptr;
    a.nqblocks = nqblocks;
    a.cache_requests = s->max_batch;
    int64_t n = rows;  // rows past the attention
    if (lq) {
      a.qrows = last;
      a.nq = cache_only ? 0 : nlast;
      n = a.nq;
    }
    trace(PH_ATTENTION, true, st);
    TF_TRY(launch_attention(a, st));
    trace(PH_ATTENTION, false, st);
    if (lq && cache_only) break;
    const void* resid = s->h0;
    if (lq) {
      TF_TRY(launch_gather_rows(s->h0, H, last, 1, nlast, H, c.act, s->hc, st));
      resid = s->hc;
    }
    QmmProblem o;
    o.mode = QMM_DENSE;
    o.epilogue = EPI_RESIDUAL;
    o.act = c.act;
    o.x = s->attn;
    o.x_stride = W;
    o.n = n;
    o.w0 = L.o;
    o.y = s->h1;
    o.y_stride = H;
    o.residual = resid;
    o.residual_stride = H;
    trace(PH_O_PROJ, true, st);
    TF_TRY(dense_qmm(s, o, n, st));
    trace(PH_O_PROJ, false, st);
    trace(PH_POST_NORM, true, st);
    TF_TRY(launch_rms_norm(s->h1, n, H, L.post_norm, c.rms_eps, c.act, s->xn, st));
    trace(PH_POST_NORM, false, st);
    tf_moe_args ma{};
    ma.x = s->xn;
    ma.residual = s->h1;
    ma.out = s->h0;
    ma.tokens = n;
    ma.hidden = H;
    ma.intermediate = c.intermediate;
    ma.experts = c.experts;
    ma.top_k = c.top_k;
    ma.act = c.act;
    ma.router.dense = nullptr;
    ma.router.affine = L.router;
    ma.gate_proj = L.gate;
    ma.up_proj = L.up;
    ma.down_proj = L.down;
    const bool capture = rows <= s->capture_rows;
    if (capture && s->route_capture) ma.indices = s->route_capture + (size_t)l * rows * c.top_k;
    // The next layer's input norm runs in this block's combine when this
    // block produced every row (not the last-query-only layer).
    MoeNextNorm nn;
    const bool fuse = l + 1 < c.layers && n == rows && H % 256 == 0 && H <= 8192;
    if (fuse) {
      nn.w = m->layers[l + 1].input_norm;
      nn.eps = c.rms_eps;
      nn.out = s->xn;
    }
    TF_TRY(moe_run(&ma, s->moe_ws, s->moe_ws_bytes, st, /*counters_zero=*/true, fuse ? &nn : nullptr));
    normed = fuse;
    if (capture && s->hidden_capture)
      TF_CUDA(cudaMemcpyAsync(static_cast<char*>(s->hidden_capture) + (size_t)l * rows * H * act_bytes(c.act), s->h0,
                              (size_t)n * H * act_bytes(c.act), cudaMemcpyDeviceToDevice, st));
  }
  return TF_OK;
}

// Final RMSNorm + lm_head of selected rows -> s->logits [n][vocab].
tf_status head_rows(tf_session* s, int64_t rows, const int32_t* sel, int64_t n, cudaStream_t st) {
  const tf_olmoe_config& c = s->m->c;
  trace(PH_FINAL_NORM, true, st);
  TF_TRY(launch_rms_norm(s->h0, rows, c.hidden, s->m->final_norm, c.rms_eps, c.act, s->xn, st));
  trace(PH_FINAL_NORM, false, st);
  QmmProblem h;
  h.mode = QMM_DENSE;
  h.epilogue = EPI_F32;
  h.act = c.act;
  h.x = s->xn;
  h.x_stride = c.hidden;
  h.x_index = sel;
  h.n = n;
  h.w0 = s->m->lm_head;
  h.y = s->logits;
  h.y_stride = c.vocab;
  trace(PH_LM_HEAD, true, st);
  TF_TRY(dense_qmm(s, h, rows, st));
  trace(PH_LM_HEAD, false, st);
  return TF_OK;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// Shared body of the decode entry points: checks, input copies, the layer
// stack and (when `head`) the final norm + lm_head into s->logits.
tf_status decode_step(tf_session* s, const int64_t* token_ids, const int32_t* positions, int32_t batch, int flags,
                      bool head, cudaStream_t st, bool* dispatched) {
  *dispatched = false;
  if (!s || !token_ids) return set_error(TF_ERR_INVALID_ARGUMENT, "decode: NULL argument");
  if (s->invalid) return refuse_invalid(s);
  if (batch <= 0 || batch > s->max_batch)
    return set_error(TF_ERR_INVALID_ARGUMENT, "decode: batch %d outside [1, %d]", batch, s->max_batch);
  if (s->cancelled.load()) return set_error(TF_ERR_CANCELLED, "session cancelled");
  const tf_olmoe_config& c = s->m->c;
  std::vector<int32_t> pos(batch);
  int max_len = 0;
  for (int b = 0; b < batch; ++b) {
    pos[b] = positions ? positions[b] : s->lengths[b];
    if (pos[b] != s->lengths[b])
      return set_error(TF_ERR_INVALID_ARGUMENT, "invalid absolute position %d for request %d (length %d)", pos[b],
                       b, s->lengths[b]);
    if (pos[b] >= s->capacity) return set_error(TF_ERR_CAPACITY, "absolute capacity exceeded (request %d)", b);
    if (pos[b] + 1 > max_len) max_len = pos[b] + 1;
    if ((flags & TF_HOST_INPUTS) && (token_ids[b] < 0 || token_ids[b] >= c.vocab))
      return set_error(TF_ERR_INVALID_ARGUMENT, "token id %lld of request %d outside the vocabulary",
                       (long long)token_ids[b], b);
  }
  *dispatched = true;
  TF_CUDA(cudaMemcpyAsync(s->ids, token_ids, (size_t)batch * 8,
                          (flags & TF_HOST_INPUTS) ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, st));
  TF_CUDA(cudaMemcpyAsync(s->pos, pos.data(), (size_t)batch * 4, cudaMemcpyHostToDevice, st));
  if (s->graphs_on && !s->tracing && !s->route_capture && !s->hidden_capture) {
    const int splits = (max_len + 255) / 256;
    tf_session::DecodeGraph& gr = s->graphs[std::make_tuple(batch, head ? 1 : 0, splits, g_qmm_path)];
    if (gr.exec || gr.eager_runs > 0) {
      TF_CUDA(cudaEventRecord(s->ev_in, st));
      TF_CUDA(cudaStreamWaitEvent(s->gstream, s->ev_in, 0));
      if (!gr.exec) {
        // The attention grid covers `splits` blocks of 256 keys; blocks past
        // a row's length exit at once, so the graph serves every length up to
        // splits * 256.
        const int graph_len = splits * 256 < s->capacity ? splits * 256 : s->capacity;
        const uint64_t c0 = launch_count();
        TF_CUDA(cudaStreamBeginCapture(s->gstream, cudaStreamCaptureModeThreadLocal));
        tf_status rc = forward_rows(s, batch, true, graph_len, s->gstream);
        if (rc == TF_OK && head) rc = head_rows(s, batch, nullptr, batch, s->gstream);
        cudaGraph_t graph = nullptr;
        const cudaError_t ce = cudaStreamEndCapture(s->gstream, &graph);
        const int64_t captured = (int64_t)(launch_count() - c0);
        add_launches(-captured);  // recorded, not run
        if (rc != TF_OK || ce != cudaSuccess) {
          if (graph) cudaGraphDestroy(graph);
          if (rc != TF_OK) return rc;
          return set_error(TF_ERR_CUDA, "decode graph capture: %s", cudaGetErrorString(ce));
        }
        const cudaError_t ie = cudaGraphInstantiate(&gr.exec, graph, 0);
        cudaGraphDestroy(graph);
        if (ie != cudaSuccess) {
          gr.exec = nullptr;
          return set_error(TF_ERR_CUDA, "decode graph instantiate: %s", cudaGetErrorString(ie));
        }
        gr.launches = captured;
      }
      TF_CUDA(cudaGraphLaunch(gr.exec, s->gstream));
      add_launches(gr.launches);
      TF_CUDA(cudaEventRecord(s->ev_out, s->gstream));
      TF_CUDA(cudaStreamWaitEvent(st, s->ev_out, 0));
      return TF_OK;
    }
    gr.eager_runs++;  // first step of this shape: kernel attributes are set, nothing is captured
  }
  TF_TRY(forward_rows(s, batch, true, max_len, st));
  if (head) TF_TRY(head_rows(s, batch, nullptr, batch, st));
  return TF_OK;
}

// The dispatched part of tf_session_prefill: input copies, the layer stack,
// the head, and the final synchronization (the host vectors are pageable),
// which is also the call's completion point for device-side failures.
tf_status prefill_dispatch(tf_session* s, int64_t rows, const int64_t* token_ids, int flags,
                           const std::vector<int32_t>& pos, const std::vector<int32_t>& req,
                           const std::vector<int32_t>& last, const std::vector<int4>& qb, int max_len,
                           int num_requests, float* last_logits, cudaStream_t st) {
  const tf_olmoe_config& c = s->m->c;
  TF_CUDA(cudaMemcpyAsync(s->ids, token_ids, (size_t)rows * 8,
                          (flags & TF_HOST_INPUTS) ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, st));
  TF_CUDA(cudaMemcpyAsync(s->pos, pos.data(), (size_t)rows * 4, cudaMemcpyHostToDevice, st));
  TF_CUDA(cudaMemcpyAsync(s->req, req.data(), (size_t)rows * 4, cudaMemcpyHostToDevice, st));
  TF_CUDA(cudaMemcpyAsync(s->last_rows, last.data(), (size_t)num_requests * 4, cudaMemcpyHostToDevice, st));
  TF_CUDA(cudaMemcpyAsync(s->qblocks, qb.data(), qb.size() * sizeof(int4), cudaMemcpyHostToDevice, st));
  TF_TRY(forward_rows(s, rows, false, max_len, st, (int)qb.size(), s->last_rows, num_requests,
                      last_logits == nullptr));
  if (last_logits) {
    // With fewer requests than rows the last layer left each request's final
    // hidden state compact in rows 0..num_requests-1.
    if (num_requests < rows)
      TF_TRY(head_rows(s, num_requests, nullptr, num_requests, st));
    else
      TF_TRY(head_rows(s, rows, s->last_rows, num_requests, st));
    TF_CUDA(cudaMemcpyAsync(last_logits, s->logits, (size_t)num_requests * c.vocab * 4,
                            (flags & TF_HOST_OUTPUT) ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, st));
  }
  TF_CUDA(cudaStreamSynchronize(st));
  return device_status();
}

}  // namespace

extern "C" {

int tf_session_decode(tf_session* s, const int64_t* token_ids, const int32_t* positions, int32_t batch,
                      float* logits, int flags, void* stream) {
  DeviceGuard g(s ? s->m->device : 0);
  TraceScope ts(s && s->tracing ? &s->tracer : nullptr);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  bool dispatched = false;
  tf_status rc = decode_step(s, token_ids, positions, batch, flags, logits != nullptr, st, &dispatched);
  if (rc != TF_OK) return dispatched ? invalidate(s, rc, st) : rc;
  if (logits) {
    const cudaError_t e = cudaMemcpyAsync(logits, s->logits, (size_t)batch * s->m->c.vocab * 4,
                                          (flags & TF_HOST_OUTPUT) ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice,
                                          st);
    if (e != cudaSuccess) return invalidate(s, set_error(TF_ERR_CUDA, "decode logits copy: %s", cudaGetErrorString(e)), st);
    if (flags & TF_HOST_OUTPUT) {
      // A host-visible completion point: device-side failures surface here.
      const cudaError_t w = cudaStreamSynchronize(st);
      if (w != cudaSuccess) return invalidate(s, set_error(TF_ERR_CUDA, "decode: %s", cudaGetErrorString(w)), st);
      rc = device_status();
      if (rc != TF_OK) return invalidate(s, rc, st);
    }
  }
  for (int b = 0; b < batch; ++b) s->lengths[b] += 1;
  return TF_OK;
}

int tf_session_decode_greedy(tf_session* s, const int64_t* token_ids, const int32_t* positions, int32_t batch,
                             int64_t* tokens, float* logits, int flags, void* stream) {
  if (!tokens) return set_error(TF_ERR_INVALID_ARGUMENT, "decode_greedy: NULL tokens");
  DeviceGuard g(s ? s->m->device : 0);
  TraceScope ts(s && s->tracing ? &s->tracer : nullptr);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  bool dispatched = false;
  tf_status rc = decode_step(s, token_ids, positions, batch, flags, true, st, &dispatched);
  if (rc != TF_OK) return dispatched ? invalidate(s, rc, st) : rc;
  const int64_t vocab = s->m->c.vocab;
  const bool host_out = (flags & TF_HOST_OUTPUT) != 0;
  rc = launch_greedy(s->logits, batch, vocab, host_out ? s->greedy : tokens, st);
  if (rc != TF_OK) return invalidate(s, rc, st);
  cudaError_t e = cudaSuccess;
  if (logits)
    e = cudaMemcpyAsync(logits, s->logits, (size_t)batch * vocab * 4,
                        host_out ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, st);
  if (e == cudaSuccess && host_out) {
    e = cudaMemcpyAsync(tokens, s->greedy, (size_t)batch * 8, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  if (e != cudaSuccess) return invalidate(s, set_error(TF_ERR_CUDA, "greedy decode: %s", cudaGetErrorString(e)), st);
  if (host_out) {
    rc = device_status();
    if (rc != TF_OK) return invalidate(s, rc, st);
  }
  for (int b = 0; b < batch; ++b) s->lengths[b] += 1;
  return TF_OK;
}

int tf_session_prefill(tf_session* s, const int32_t* requests, const int32_t* token_counts, int32_t num_requests,
                       const int64_t* token_ids, float* last_logits, int flags, void* stream) {
  if (!s || !requests || !token_counts || !token_ids)
    return set_error(TF_ERR_INVALID_ARGUMENT, "prefill: NULL argument");
  if (s->invalid) return refuse_invalid(s);
  if (num_requests <= 0 || num_requests > s->max_batch)
    return set_error(TF_ERR_INVALID_ARGUMENT, "prefill: %d requests outside [1, %d]", num_requests, s->max_batch);
  if (s->cancelled.load()) return set_error(TF_ERR_CANCELLED, "session cancelled");
  const tf_olmoe_config& c = s->m->c;
  std::vector<int32_t> pos, req, last(num_requests);
  std::vector<int4> qb;
  std::vector<char> seen(s->max_batch, 0);
  int max_len = 0;
  for (int i = 0; i < num_requests; ++i) {
    const int r = requests[i], n = token_counts[i];
    if (r < 0 || r >= s->max_batch || seen[r])
      return set_error(TF_ERR_INVALID_ARGUMENT, "prefill: request %d invalid or repeated", r);
    seen[r] = 1;
    if (n <= 0) return set_error(TF_ERR_INVALID_ARGUMENT, "prefill: request %d has %d tokens", r, n);
    const int start = s->lengths[r];
    if ((int64_t)start + n > s->capacity) return set_error(TF_ERR_CAPACITY, "absolute capacity exceeded");
    // query blocks of up to kPrefillQueryBlock rows of this request (tiled
    // prefill attention)
    for (int b0 = 0; b0 < n; b0 += kPrefillQueryBlock)
      qb.push_back(make_int4((int)pos.size() + b0, n - b0 < kPrefillQueryBlock ? n - b0 : kPrefillQueryBlock, r,
                             start + b0));
    for (int t = 0; t < n; ++t) {
      pos.push_back(start + t);
      req.push_back(r);
    }
    last[i] = (int32_t)pos.size() - 1;
    if (start + n > max_len) max_len = start + n;
  }
  // Blocks with the most keys first, so that the longest ones do not start
  // in the last wave.
  std::stable_sort(qb.begin(), qb.end(), [](const int4& x, const int4& y) { return x.w + x.y > y.w + y.y; });
  const int64_t rows = (int64_t)pos.size();
  if (rows > s->max_rows)
    return set_error(TF_ERR_CAPACITY, "prefill: %lld rows exceed the session's %d", (long long)rows, s->max_rows);
  if (flags & TF_HOST_INPUTS)
    for (int64_t i = 0; i < rows; ++i)
      if (token_ids[i] < 0 || token_ids[i] >= c.vocab)
        return set_error(TF_ERR_INVALID_ARGUMENT, "prefill: token id %lld at row %lld outside the vocabulary",
                         (long long)token_ids[i], (long long)i);
  DeviceGuard g(s->m->device);
  TraceScope ts(s->tracing ? &s->tracer : nullptr);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const tf_status rc = prefill_dispatch(s, rows, token_ids, flags, pos, req, last, qb, max_len, num_requests,
                                        last_logits, st);
  // Everything after the first copy counts as dispatched.
  if (rc != TF_OK) return invalidate(s, rc, st);
  for (int i = 0; i < num_requests; ++i) s->lengths[requests[i]] += token_counts[i];
  return TF_OK;
}

int tf_session_prefill_chunked(tf_session* s, int32_t request, const int64_t* token_ids, int64_t count,
                               int32_t chunk_tokens, float* last_logits, int flags, void* stream) {
  if (!s || !token_ids) return set_error(TF_ERR_INVALID_ARGUMENT, "chunked prefill: NULL argument");
  if (!(flags & TF_HOST_INPUTS))
    return set_error(TF_ERR_INVALID_ARGUMENT, "chunked prefill: token ids must be host memory (validated first)");
  if (request < 0 || request >= s->max_batch)
    return set_error(TF_ERR_INVALID_ARGUMENT, "chunked prefill: request %d outside [0, %d)", request, s->max_batch);
  if (count <= 0) return set_error(TF_ERR_INVALID_ARGUMENT, "chunked prefill: %lld tokens", (long long)count);
  if (chunk_tokens <= 0 || chunk_tokens > s->max_rows)
    return set_error(TF_ERR_INVALID_ARGUMENT, "chunked prefill: chunk of %d tokens outside [1, %d]", chunk_tokens,
                     s->max_rows);
  if ((int64_t)s->lengths[request] + count > s->capacity)
    return set_error(TF_ERR_CAPACITY, "absolute capacity exceeded");
  const int64_t vocab = s->m->c.vocab;
  // Every input is validated before the first chunk is dispatched.
  for (int64_t i = 0; i < count; ++i)
    if (token_ids[i] < 0 || token_ids[i] >= vocab)
      return set_error(TF_ERR_INVALID_ARGUMENT, "chunked prefill: token %lld at %lld outside the vocabulary",
                       (long long)token_ids[i], (long long)i);
  for (int64_t off = 0; off < count; off += chunk_tokens) {
    const int32_t n = (int32_t)((count - off) < chunk_tokens ? (count - off) : chunk_tokens);
    const bool last = off + n == count;
    // Intermediate chunks only extend the KV cache (no logits).
    const int rc = tf_session_prefill(s, &request, &n, 1, token_ids + off, last ? last_logits : nullptr, flags, stream);
    if (rc != TF_OK) return rc;
  }
  if (last_logits && (flags & TF_HOST_OUTPUT))
    for (int64_t i = 0; i < vocab; ++i)
      if (!std::isfinite(last_logits[i])) return set_error(TF_ERR_STATE, "non-finite final prefill logits");
  return TF_OK;
}

int tf_trace_phases(void) { return PH_COUNT; }

const char* tf_trace_phase_name(int phase) {
  return (phase >= 0 && phase < PH_COUNT) ? kPhaseNames[phase] : "";
}

int tf_session_graphs(tf_session* s, int enable) {
  if (!s) return set_error(TF_ERR_INVALID_ARGUMENT, "NULL session");
  if (enable && (!s->gstream || !s->ev_in || !s->ev_out))
    return set_error(TF_ERR_UNSUPPORTED, "graph stream/events could not be created");
  s->graphs_on = enable != 0;
  return TF_OK;
}

int tf_session_capture(tf_session* s, int32_t* indices, void* hidden, int64_t max_rows) {
  if (!s) return set_error(TF_ERR_INVALID_ARGUMENT, "session is NULL");
  if ((indices || hidden) && max_rows <= 0) return set_error(TF_ERR_INVALID_ARGUMENT, "capture: max_rows must be positive");
  s->route_capture = indices;
  s->hidden_capture = hidden;
  s->capture_rows = (indices || hidden) ? max_rows : 0;
  return TF_OK;
}

int tf_session_trace(tf_session* s, int enable) {
  if (!s) return set_error(TF_ERR_INVALID_ARGUMENT, "session is NULL");
  s->tracing = enable != 0;
  return TF_OK;
}

int tf_session_trace_read(tf_session* s, float* total_ms, int32_t* counts) {
  if (!s || !total_ms || !counts) return set_error(TF_ERR_INVALID_ARGUMENT, "NULL argument");
  for (int p = 0; p < PH_COUNT; ++p) {
    total_ms[p] = 0.f;
    counts[p] = 0;
  }
  DeviceGuard g(s->m->device);
  for (auto& pr : s->tracer.pairs) {
    TF_CUDA(cudaEventSynchronize(pr.b));
    float ms = 0.f;
    TF_CUDA(cudaEventElapsedTime(&ms, pr.a, pr.b));
    total_ms[pr.phase] += ms;
    counts[pr.phase] += 1;
  }
  s->tracer.recycle();
  return TF_OK;
}

}  // extern "C"
