// Weighted top-k combine + residual.
//
// Restates MLXNativeGraniteMoEPrefill.h:688-695 (out[inverse], multiply by the
// gates and sum over k, each in the activation dtype) and the layer residual
// (tools/export/export_native_olmoe_target.py:218, 227):
//   out = act(residual + act(sum_k act(y_k * g_k)))
// with the fp32 sum taken in k order starting from the k = 0 product
// (bit-identical to oracle/olmoe.py: combine).
#include "common.cuh"
#include "internal.h"

namespace tf {

template <typename T, bool NORM>
__global__ void __launch_bounds__(256)
    combine_kernel(const T* __restrict__ y, const int32_t* __restrict__ inverse,
                   const T* __restrict__ gates, const T* __restrict__ residual, int K, int H,
                   T* __restrict__ out, const __half* __restrict__ norm_w, float eps, T* __restrict__ norm_out) {
  const int cpr = (H / 8 + blockDim.x - 1) / blockDim.x;  // blocks per token row
  const int64_t t = blockIdx.x / cpr;
  const int c = (int)(blockIdx.x % cpr) * blockDim.x + threadIdx.x;  // 8-element chunk
  if (!NORM && 8 * c >= H) return;
  float acc[8];
  for (int k = 0; k < K; ++k) {
    const int64_t slot = inverse[t * K + k];
    const float g = to_f(gates[t * K + k]);
    float v[8];
    unpack8<T>(ld_v4(y + slot * H + 8 * c), v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float pr = round_act<T>(__fmul_rn(v[i], g));
      acc[i] = k == 0 ? pr : __fadd_rn(acc[i], pr);
    }
  }
  float r[8];
  unpack8<T>(ld_v4(residual + t * H + 8 * c), r);
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = round_act<T>(__fadd_rn(r[i], round_act<T>(acc[i])));
  *reinterpret_cast<uint4*>(out + t * H + 8 * c) = pack8<T>(acc);
  if (NORM) {
    // The next layer's input RMSNorm of this row, in rms_norm_kernel's
    // order (one thread per 8-element chunk, warp butterflies, warp totals
    // added in warp order by thread 0), on the stored (act-rounded) values.
    __shared__ float warp_tot[32];
    __shared__ float scale_s;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float v = warp_sum_butterfly(chunk_sumsq8(acc));
    if (lane == 0) warp_tot[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
      float tot = warp_tot[0];
      for (int i = 1; i < (int)(blockDim.x >> 5); ++i) tot = __fadd_rn(tot, warp_tot[i]);
      scale_s = rms_scale(tot, H, eps);
    }
    __syncthreads();
    const float rs = scale_s;
    const uint4 wv = ld_v4(norm_w + 8 * c);
    const __half* wh = reinterpret_cast<const __half*>(&wv);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(__fmul_rn(acc[i], rs), __half2float(wh[i]));
    *reinterpret_cast<uint4*>(norm_out + t * H + 8 * c) = pack8<T>(o);
  }
}

tf_status launch_combine(const void* y_sorted, const int32_t* inverse, const void* gates,
                         const void* residual, int64_t tokens, int k, int hidden, int act,
                         void* out, cudaStream_t s, const void* norm_w, float eps, void* norm_out) {
  if (tokens == 0) return TF_OK;
  if (norm_out) {
    // One block of hidden / 8 threads per row (rms_norm_kernel's shape).
    if (hidden % 256 || hidden > 8192)
      return set_error(TF_ERR_UNSUPPORTED, "combine+norm: hidden %d", hidden);
    const unsigned threads = (unsigned)(hidden / 8);
    if (act == TF_DTYPE_F16)
      combine_kernel<__half, true><<<(unsigned)tokens, threads, 0, s>>>(
          (const __half*)y_sorted, inverse, (const __half*)gates, (const __half*)residual, k, hidden,
          (__half*)out, (const __half*)norm_w, eps, (__half*)norm_out);
    else
      combine_kernel<__nv_bfloat16, true><<<(unsigned)tokens, threads, 0, s>>>(
          (const __nv_bfloat16*)y_sorted, inverse, (const __nv_bfloat16*)gates, (const __nv_bfloat16*)residual, k,
          hidden, (__nv_bfloat16*)out, (const __half*)norm_w, eps, (__nv_bfloat16*)norm_out);
    return check_launch("combine_norm");
  }
  const unsigned grid = (unsigned)(tokens * ((hidden / 8 + 255) / 256));
  if (act == TF_DTYPE_F16)
    combine_kernel<__half, false><<<grid, 256, 0, s>>>((const __half*)y_sorted, inverse, (const __half*)gates,
                                                       (const __half*)residual, k, hidden, (__half*)out, nullptr,
                                                       0.f, nullptr);
  else
    combine_kernel<__nv_bfloat16, false><<<grid, 256, 0, s>>>(
        (const __nv_bfloat16*)y_sorted, inverse, (const __nv_bfloat16*)gates, (const __nv_bfloat16*)residual, k,
        hidden, (__nv_bfloat16*)out, nullptr, 0.f, nullptr);
  return check_launch("combine");
}

// Row gather in the activation dtype (16-byte vectors): y[i] = x[idx[i] / div]
// (the last rows of a prefill's requests as a compact batch for the last
// layer's queries; the routed rows of an expert-parallel dispatch).
__global__ void gather_rows_kernel(const uint4* __restrict__ x, int64_t x_stride16, const int32_t* __restrict__ idx,
                                   int div, int64_t n, int width16, uint4* __restrict__ y) {
  const int64_t i = blockIdx.x;
  if (i >= n) return;
  const int64_t src = idx[i] / div;
  for (int c = threadIdx.x; c < width16; c += blockDim.x) y[i * width16 + c] = x[src * x_stride16 + c];
}

tf_status launch_gather_rows(const void* x, int64_t x_stride, const int32_t* idx, int div, int64_t n, int width,
                             int act, void* y, cudaStream_t s) {
  if (n == 0) return TF_OK;
  const int eb = act_bytes(act);
  if ((width * eb) % 16 || (x_stride * eb) % 16) return set_error(TF_ERR_SHAPE, "gather_rows: width %d", width);
  if (n > 2147483647) return set_error(TF_ERR_UNSUPPORTED, "gather_rows: too many rows");
  gather_rows_kernel<<<(unsigned)n, 128, 0, s>>>((const uint4*)x, x_stride * eb / 16, idx, div, n,
                                                 width * eb / 16, (uint4*)y);
  return check_launch("gather_rows");
}

}  // namespace tf
