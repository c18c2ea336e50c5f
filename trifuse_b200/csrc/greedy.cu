// Greedy next-token selection on the device.
//
// Restates the reference's greedy submission (patches/executorch.patch:
// 1350-1353): token = all(isfinite(logits)) ? int64(argmax(logits)) : -1, per
// row of fp32 logits; argmax takes the lowest index among equal maxima (the
// first occurrence).  The token stays in device memory so the next decode
// step can consume it before the host reads it (one-ahead submission,
// src/apple/TFETResidentSession.mm:1113-1189); the consumer reads a negative
// token as 0 (the reference's maximum(token, 0), executorch.patch:1125-1126).
#include "common.cuh"
#include "internal.h"

namespace tf {

namespace {

constexpr int kGreedyThreads = 512;

// (value, index) max with ties to the lower index.
__device__ __forceinline__ void better(float& v, int64_t& i, float v2, int64_t i2) {
  if (v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}

__global__ void __launch_bounds__(kGreedyThreads)
    greedy_kernel(const float* __restrict__ logits, int64_t vocab, int64_t* __restrict__ tokens) {
  const float* row = logits + (int64_t)blockIdx.x * vocab;
  float best = -INFINITY;
  int64_t at = vocab;  // past the end until a finite value is seen
  int bad = 0;
  for (int64_t j = threadIdx.x; j < vocab; j += blockDim.x) {
    const float v = row[j];
    if (!isfinite(v)) {
      bad = 1;
      continue;
    }
    better(best, at, v, j);
  }
  bad = __syncthreads_or(bad);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float v2 = __shfl_xor_sync(0xffffffffu, best, off);
    const int64_t i2 = __shfl_xor_sync(0xffffffffu, at, off);
    better(best, at, v2, i2);
  }
  __shared__ float sv[kGreedyThreads / 32];
  __shared__ int64_t si[kGreedyThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = at;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kGreedyThreads / 32; ++w) better(best, at, sv[w], si[w]);
    tokens[blockIdx.x] = (bad || at >= vocab) ? -1 : at;
  }
}

}  // namespace

tf_status launch_greedy(const float* logits, int64_t rows, int64_t vocab, int64_t* tokens, cudaStream_t s) {
  if (rows == 0) return TF_OK;
  if (rows > 2147483647) return set_error(TF_ERR_UNSUPPORTED, "greedy: too many rows");
  greedy_kernel<<<(unsigned)rows, kGreedyThreads, 0, s>>>(logits, vocab, tokens);
  return check_launch("greedy");
}

}  // namespace tf
