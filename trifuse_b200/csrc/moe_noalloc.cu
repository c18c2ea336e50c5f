// tf_moe_forward_noalloc: the MoE block for callers that must not allocate.
//
// Some callers cannot call cudaMalloc at all while they run this block:
// a host framework's execute callback whose device memory was planned ahead
// of time (the ExecuTorch delegate this path replaces owns every buffer and
// gives the backend no allocation hook), or a latency-critical serving loop
// where cudaMalloc / cudaFree may synchronize the whole device and stall the
// other streams.  For them this entry point takes only the block's inputs
// and outputs and runs the same computation as tf_moe_forward, with the
// scratch taken from one fixed buffer compiled into the library.
//
// The buffer is a file-scope __device__ array: every GPU that loads this
// library holds kScratchBytes of it until the process exits.  In host code
// the array's name is only a host-side stand-in, so its device address is
// looked up once per device (cudaGetSymbolAddress with that device current)
// on the first call made on that device, and passed to the kernels.  Make
// that first call before any stream capture.  The address is kept for the
// life of the process: after a device reset the module (and the array) may
// load elsewhere, so this entry must not be used across one.  With lazy
// module loading the first call per device and batch shape may load kernel
// modules (the driver allocates for them); a warm-up call, or
// CUDA_MODULE_LOADING=EAGER, moves that out of the caller's critical path.  The address is kept for the
// life of the process: after a device reset the module (and the array) may
// load elsewhere, so this entry must not be used across one.  With lazy
// module loading the first call per device and batch shape may load kernel
// modules (the driver allocates for them); a warm-up call, or
// CUDA_MODULE_LOADING=EAGER, moves that out of the caller's critical path.
//
// Every call shares the one buffer and leaves its contents behind; nothing
// in it has to start at zero, because each call writes every scratch byte
// it later reads.  Two calls that overlap on the GPU (different streams, or
// different host threads) race on the buffer: serialize them.
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace {

// Covers one decode step of up to 64 tokens at OLMoE-1B-7B geometry
// (hidden 2048, intermediate 1024, 64 experts, top-8, f16 or bf16):
// about 5 MiB of route buffers, expert intermediates and f16 operand copies.
constexpr size_t kScratchBytes = TF_MOE_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_moe_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

tf_status scratch_on_current_device(void** out) {
  int dev = -1;
  TF_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return tf::set_error(TF_ERR_UNSUPPORTED, "tf_moe_forward_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_moe_scratch);
    if (e != cudaSuccess || !p)
      return tf::set_error(TF_ERR_CUDA, "tf_moe_forward_noalloc: cudaGetSymbolAddress on device %d: %s", dev,
                           cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return TF_OK;
}

}  // namespace

extern "C" int tf_moe_forward_noalloc(const tf_moe_args* args, void* stream) {
  size_t need = 0;
  // Same admission as tf_moe_forward (geometry, dtypes, pointers).
  TF_TRY((tf_status)tf_moe_workspace_size(args, &need));
  // This entry runs without the tensor-core split buffers (each tile on one
  // block), so it needs only the block's own scratch.
  need = tf::moe_workspace_bytes(args, false);
  if (args->tokens > TF_MOE_NOALLOC_MAX_TOKENS)
    return tf::set_error(TF_ERR_CAPACITY,
                         "tf_moe_forward_noalloc: %lld tokens exceed the fixed buffer's limit of %d; "
                         "call tf_moe_forward with a workspace instead",
                         (long long)args->tokens, TF_MOE_NOALLOC_MAX_TOKENS);
  if (need > kScratchBytes)
    return tf::set_error(TF_ERR_CAPACITY,
                         "tf_moe_forward_noalloc: this call needs %zu bytes of scratch but the fixed buffer "
                         "holds %zu (up to 64 tokens at hidden 2048 / intermediate 1024 / 64 experts / top-8); "
                         "call tf_moe_forward with a workspace instead",
                         need, kScratchBytes);
  if (args->tokens == 0) return TF_OK;
  void* ws = nullptr;
  TF_TRY(scratch_on_current_device(&ws));
  return tf_moe_forward(args, ws, kScratchBytes, stream);
}
