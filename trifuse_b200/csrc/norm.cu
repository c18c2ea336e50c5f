// RMSNorm and 4-bit embedding gather.
//
// rms_norm restates fast::rms_norm as used at MLXNativeGraniteMoEPrefill.h:434,
// 451-452, 486, 490 with the fixed reduction order documented in the oracle
// (oracle/olmoe.py: row_sumsq): thread t owns the 8-element chunk t, warps
// combine with the xor butterfly, warp totals are added left to right.
#include "common.cuh"
#include "internal.h"

namespace tf {

// Block of width/8 threads (one 16-byte chunk each), one row per block.
template <typename T>
__global__ void __launch_bounds__(1024) rms_norm_kernel(const T* __restrict__ x, int width,
                                                        const __half* __restrict__ w, float eps,
                                                        T* __restrict__ y) {
  __shared__ float warp_tot[32];
  __shared__ float scale_s;
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5;
  const uint4 xv = ld_v4(x + row * width + 8 * t);
  float xf[8];
  unpack8<T>(xv, xf);
  float v = warp_sum_butterfly(chunk_sumsq8(xf));
  if (lane == 0) warp_tot[warp] = v;
  __syncthreads();
  if (t == 0) {
    float tot = warp_tot[0];
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) tot = __fadd_rn(tot, warp_tot[i]);
    scale_s = rms_scale(tot, width, eps);
  }
  __syncthreads();
  const float r = scale_s;
  const uint4 wv = ld_v4(w + 8 * t);
  const __half* wh = reinterpret_cast<const __half*>(&wv);
  float out[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) out[i] = __fmul_rn(__fmul_rn(xf[i], r), __half2float(wh[i]));
  *reinterpret_cast<uint4*>(y + row * width + 8 * t) = pack8<T>(out);
}

tf_status launch_rms_norm(const void* x, int64_t rows, int width, const void* w, float eps,
                          int act, void* y, cudaStream_t s) {
  if (rows == 0) return TF_OK;
  const int threads = width / 8;
  if (act == TF_DTYPE_F16)
    rms_norm_kernel<__half><<<(unsigned)rows, threads, 0, s>>>(
        (const __half*)x, width, (const __half*)w, eps, (__half*)y);
  else
    rms_norm_kernel<__nv_bfloat16><<<(unsigned)rows, threads, 0, s>>>(
        (const __nv_bfloat16*)x, width, (const __half*)w, eps, (__nv_bfloat16*)y);
  return check_launch("rms_norm");
}

// Embedding: row ids[n] of the packed table, dequantized as fp16(code*s + b)
// (native_affine_ops.py:29-36, 77-87) and converted to the output dtype.
// One thread per packed word (8 values).
__device__ int g_embed_error = 0;  // 6: a token id past the embedding table

template <typename T>
__global__ void embedding_kernel(const int64_t* __restrict__ ids, const uint32_t* __restrict__ q,
                                 const __half* __restrict__ sc, const __half* __restrict__ bi,
                                 int width, int64_t rows, T* __restrict__ y) {
  const int bpr = (width / 8 + blockDim.x - 1) / blockDim.x;  // blocks per row
  const int64_t n = blockIdx.x / bpr;
  const int word = (int)(blockIdx.x % bpr) * blockDim.x + threadIdx.x;
  if (word >= width / 8) return;
  // A negative id (the greedy "non-finite logits" token fed back on the
  // device) reads row 0, as the reference's maximum(token, 0); an id past the
  // table reads row 0 too and records error code 6 (tf_device_error).
  int64_t row = ids[n];
  if (row >= rows) {
    if (word == 0) atomicCAS(&g_embed_error, 0, 6);
    row = 0;
  }
  if (row < 0) row = 0;
  const uint32_t wv = q[row * (width / 8) + word];
  const int g = word / 8;
  const float s = __half2float(sc[row * (width / 64) + g]);
  const float b = __half2float(bi[row * (width / 64) + g]);
  float out[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float code = (float)((wv >> (4 * j)) & 0xFu);
    out[j] = __half2float(__float2half_rn(__fadd_rn(__fmul_rn(code, s), b)));
  }
  *reinterpret_cast<uint4*>(y + n * width + 8 * word) = pack8<T>(out);
}

tf_status launch_embedding(const int64_t* ids, int64_t n, const tf_affine_weight& t, int out,
                           void* y, cudaStream_t s) {
  if (n == 0) return TF_OK;
  const int width = t.in_features;
  const unsigned grid = (unsigned)(n * ((width / 8 + 255) / 256));
  if (out == TF_DTYPE_F16)
    embedding_kernel<__half><<<grid, 256, 0, s>>>(ids, t.q, (const __half*)t.scales,
                                                   (const __half*)t.biases, width, t.out_features,
                                                   (__half*)y);
  else
    embedding_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        ids, t.q, (const __half*)t.scales, (const __half*)t.biases, width, t.out_features,
        (__nv_bfloat16*)y);
  return check_launch("embedding");
}

int read_embed_error(bool clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_embed_error, sizeof(int));
  if (clear) {
    const int z = 0;
    cudaMemcpyToSymbol(g_embed_error, &z, sizeof(int));
  }
  return v;
}

// True when this library's sm_100a image loads on the current device.
bool kernel_image_ok() {
  cudaFuncAttributes attr;
  return cudaFuncGetAttributes(&attr, rms_norm_kernel<__half>) == cudaSuccess;
}

}  // namespace tf
