// OLMoE router: GEMV + softmax + stable top-k, and the stable route sort.
//
// Restates (file:line relative to the TriFuse root):
//  - linear(x, layer.router)          MLXNativeGraniteMoEPrefill.h:631
//  - olmoe_route / Metal router        overlays/executorch/backends/mlx/runtime/
//                                      MLXOLMoERouter.h:19-120
//  - native_olmoe_softmax / topk       native_affine_ops.py:128-153
//  - route sort (argsort + inverse)    MLXNativeGraniteMoEPrefill.h:666-684
//
// Every fp32 step is explicitly rounded so the result is
// bit-identical to oracle/olmoe.py (router_logits_*, olmoe_softmax,
// olmoe_topk): the dot product uses the chunk order "lane l owns 8-element
// chunks l + 32j", the softmax uses exp in double rounded to fp32, and the
// rank compares the act-rounded probabilities (NaN last, ties to lower id).
#include <math.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "internal.h"

namespace tf {

constexpr int kRouterWarps = 4;

// Ranks and writes the top-k of one token.  la0/la1: act-rounded logits of
// experts lane and lane+32 (ignored when >= E).
template <typename T>
__device__ __forceinline__ void route_token(int lane, float la0, float la1, int E, int K,
                                            int64_t t, T* probs, int32_t* idx, T* gates) {
  const bool v0 = lane < E, v1 = lane + 32 < E;
  float m = -INFINITY;
  if (v0) m = fmaxf(m, la0);
  if (v1) m = fmaxf(m, la1);
  m = warp_max(m);
  float e0 = 0.f, e1 = 0.f, part = 0.f;
  if (v0) {
    e0 = __double2float_rn(exp((double)__fsub_rn(la0, m)));
    part = __fadd_rn(part, e0);
  }
  if (v1) {
    e1 = __double2float_rn(exp((double)__fsub_rn(la1, m)));
    part = __fadd_rn(part, e1);
  }
  const float sum = warp_sum_butterfly(part);
  const float p0 = round_act<T>(__fdiv_rn(e0, sum));
  const float p1 = round_act<T>(__fdiv_rn(e1, sum));
  if (probs) {
    if (v0) probs[t * E + lane] = from_f<T>(p0);
    if (v1) probs[t * E + lane + 32] = from_f<T>(p1);
  }
  if (!idx) return;
  int r0 = 0, r1 = 0;
  const bool n0 = isnan(p0), n1 = isnan(p1);
  for (int j = 0; j < E; ++j) {
    const float o = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
    const bool on = isnan(o);
    // MLXOLMoERouter.h:67-78: before = other ranks strictly first; equal
    // values (or both NaN) keep increasing expert id.
    const bool before0 = !on && (n0 || o > p0);
    const bool eq0 = (on && n0) || (!on && !n0 && o == p0);
    r0 += (before0 || (eq0 && j < lane)) ? 1 : 0;
    const bool before1 = !on && (n1 || o > p1);
    const bool eq1 = (on && n1) || (!on && !n1 && o == p1);
    r1 += (before1 || (eq1 && j < lane + 32)) ? 1 : 0;
  }
  if (v0 && r0 < K) {
    idx[t * K + r0] = lane;
    if (gates) gates[t * K + r0] = from_f<T>(p0);
  }
  if (v1 && r1 < K) {
    idx[t * K + r1] = lane + 32;
    if (gates) gates[t * K + r1] = from_f<T>(p1);
  }
}

// Router GEMV.  A block of 8 warps owns TPC tokens; warp w computes experts
// w, w + 8, ... for all of them, so each weight chunk is decoded once per
// block and reused across its tokens.  Per (token, expert) the arithmetic is
// the fixed order above: lane l accumulates chunks l + 32j (j outer, the 8
// elements of a chunk inner) with separate fp32 multiply and add, then the
// xor butterfly.  The logits go through shared memory to one warp per token
// for the softmax / rank.  J = hidden / 256.
constexpr int kRouterBlockWarps = 8;

template <typename T, bool DENSE, int J, int TPC>
__global__ void __launch_bounds__(kRouterBlockWarps * 32)
    router_kernel(const T* __restrict__ x, int64_t tokens, const T* __restrict__ wd,
                  const uint32_t* __restrict__ wq, const __half* __restrict__ ws,
                  const __half* __restrict__ wb, int E, int K, T* logits, int32_t* idx, T* gates) {
  constexpr int H = J * 256;
  __shared__ float xs[TPC][H];
  __shared__ float ls[TPC][64];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t t0 = (int64_t)blockIdx.x * TPC;
  for (int i = threadIdx.x; i < TPC * H / 8; i += blockDim.x) {
    const int t = i / (H / 8), c = i % (H / 8);
    float f[8];
    if (t0 + t < tokens) {
      unpack8<T>(ld_v4(x + (t0 + t) * H + 8 * c), f);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) xs[t][8 * c + k] = f[k];
  }
  __syncthreads();
  for (int e = warp; e < E; e += kRouterBlockWarps) {
    float acc[TPC];
#pragma unroll
    for (int t = 0; t < TPC; ++t) acc[t] = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      float wf[8];
      if (DENSE) {
        unpack8<T>(ld_v4(wd + (int64_t)e * H + 8 * c), wf);
      } else {
        const uint32_t word = wq[(int64_t)e * (H / 8) + c];
        const float sc = __half2float(ws[(int64_t)e * (H / 64) + c / 8]);
        const float bi = __half2float(wb[(int64_t)e * (H / 64) + c / 8]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float code = (float)((word >> (4 * i)) & 0xFu);
          wf[i] = __half2float(__float2half_rn(__fadd_rn(__fmul_rn(code, sc), bi)));
        }
      }
#pragma unroll
      for (int t = 0; t < TPC; ++t) {
        const float* xt = &xs[t][8 * c];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[t] = __fadd_rn(acc[t], __fmul_rn(xt[i], wf[i]));
      }
    }
#pragma unroll
    for (int t = 0; t < TPC; ++t) {
      const float la = round_act<T>(warp_sum_butterfly(acc[t]));
      if (lane == 0) {
        ls[t][e] = la;
        if (logits && t0 + t < tokens) logits[(t0 + t) * E + e] = from_f<T>(la);
      }
    }
  }
  __syncthreads();
  if (idx && warp < TPC && t0 + warp < tokens) {
    const float la0 = lane < E ? ls[warp][lane] : 0.f;
    const float la1 = lane + 32 < E ? ls[warp][lane + 32] : 0.f;
    route_token<T>(lane, la0, la1, E, K, t0 + warp, (T*)nullptr, idx, gates);
  }
}

// Router for prefill-sized batches: a block of kRouterWideWarps warps owns
// kRouterWideTokens tokens, so each weight chunk is decoded once per 8
// tokens (8 rather than 16: 66 KB of shared memory and 120 registers let two
// blocks share an SM, measured 17% faster); each warp takes
// kRouterWideExperts experts at a time, so each
// activation pair read from shared memory feeds four experts; the per-token
// arithmetic runs on packed fp32 pairs
// (mul.rn.f32x2 / add.rn.f32x2: two tokens' products and sums per
// instruction, each lane of the pair rounded as the scalar op).  The order
// per (token, expert) is router_kernel's: lane l, chunks l + 32j (j outer),
// the 8 elements of a chunk in order, separate multiply and add, then the
// xor butterfly, so the logits are bit-identical.  Shared layout: token pair
// p, element pair q of chunk c at float4 [(4p + q) * C + c] = (x[2p][8c+2q],
// x[2p+1][8c+2q], x[2p][8c+2q+1], x[2p+1][8c+2q+1]); a warp's lanes read 32
// consecutive float4 (no bank conflicts).
constexpr int kRouterWideWarps = 8;
constexpr int kRouterWideTokens = 8;
constexpr int kRouterWideExperts = 4;

__device__ __forceinline__ uint64_t f32x2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f32x2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
// acc + x * w, two lanes, each rounded as __fmul_rn then __fadd_rn.
__device__ __forceinline__ uint64_t f32x2_mul_add(uint64_t acc, uint64_t x, uint64_t w) {
  uint64_t prod, r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(prod) : "l"(x), "l"(w));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(acc), "l"(prod));
  return r;
}

template <int J>
constexpr size_t router_wide_smem() {
  return (size_t)kRouterWideTokens * J * 256 * sizeof(float) + (size_t)kRouterWideTokens * 64 * sizeof(float);
}

template <typename T, bool DENSE, int J>
__global__ void __launch_bounds__(kRouterWideWarps * 32, 2)
    router_wide_kernel(const T* __restrict__ x, int64_t tokens, const T* __restrict__ wd,
                       const uint32_t* __restrict__ wq, const __half* __restrict__ ws,
                       const __half* __restrict__ wb, int E, int K, T* logits, int32_t* idx, T* gates) {
  constexpr int H = J * 256, C = H / 8, TP = kRouterWideTokens / 2;
  extern __shared__ float4 xs4[];
  float* xsf = reinterpret_cast<float*>(xs4);
  float* ls = xsf + (size_t)kRouterWideTokens * H;  // [tokens][64]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t t0 = (int64_t)blockIdx.x * kRouterWideTokens;
  static_assert(kRouterWideTokens * C % (kRouterWideWarps * 32) == 0, "whole fill rounds");
#pragma unroll
  for (int i = threadIdx.x; i < kRouterWideTokens * C; i += kRouterWideWarps * 32) {
    const int t = i / C, c = i % C;
    float f[8];
    if (t0 + t < tokens) {
      unpack8<T>(ld_v4(x + (t0 + t) * H + 8 * c), f);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = 0.f;
    }
    const int pr = t >> 1, sl = t & 1;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float* d = xsf + ((size_t)(4 * pr + q) * C + c) * 4;
      d[sl] = f[2 * q];
      d[2 + sl] = f[2 * q + 1];
    }
  }
  __syncthreads();
  // A warp computes kRouterWideExperts experts at once, so each activation
  // pair read from shared memory feeds that many products (shared-memory
  // bandwidth, not the FP pipes, bounds the one-expert-per-warp form).
  constexpr int EB = kRouterWideExperts;
  for (int e0 = warp * EB; e0 < E; e0 += kRouterWideWarps * EB) {
    uint64_t acc[EB][TP];
#pragma unroll
    for (int k = 0; k < EB; ++k)
#pragma unroll
      for (int p = 0; p < TP; ++p) acc[k][p] = 0ull;  // (+0.f, +0.f)
    // The next chunk's weights are loaded while this one is multiplied.
    uint4 nd[EB];
    uint32_t nword[EB];
    __half nsc[EB], nbi[EB];
    auto fetch = [&](int j) {
      const int c = lane + 32 * j;
#pragma unroll
      for (int k = 0; k < EB; ++k) {
        const int e = e0 + k < E ? e0 + k : E - 1;  // past E: a valid row, results dropped
        if (DENSE) {
          nd[k] = ld_v4(wd + (int64_t)e * H + 8 * c);
        } else {
          nword[k] = wq[(int64_t)e * (H / 8) + c];
          nsc[k] = ws[(int64_t)e * (H / 64) + c / 8];
          nbi[k] = wb[(int64_t)e * (H / 64) + c / 8];
        }
      }
    };
    fetch(0);
#pragma unroll 1
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      uint64_t w2[EB][8];
#pragma unroll
      for (int k = 0; k < EB; ++k) {
        float wf[8];
        if (DENSE) {
          unpack8<T>(nd[k], wf);
        } else {
          const uint32_t word = nword[k];
          const float sc = __half2float(nsc[k]);
          const float bi = __half2float(nbi[k]);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float code = (float)((word >> (4 * i)) & 0xFu);
            wf[i] = __half2float(__float2half_rn(__fadd_rn(__fmul_rn(code, sc), bi)));
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) w2[k][i] = f32x2_pack(wf[i], wf[i]);
      }
      if (j + 1 < J) fetch(j + 1);
#pragma unroll
      for (int p = 0; p < TP; ++p) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = xs4[(size_t)(4 * p + q) * C + c];
          const uint64_t lo = f32x2_pack(v.x, v.y), hi = f32x2_pack(v.z, v.w);
#pragma unroll
          for (int k = 0; k < EB; ++k) {
            acc[k][p] = f32x2_mul_add(acc[k][p], lo, w2[k][2 * q]);
            acc[k][p] = f32x2_mul_add(acc[k][p], hi, w2[k][2 * q + 1]);
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < EB; ++k) {
      const int e = e0 + k;
#pragma unroll
      for (int p = 0; p < TP; ++p) {
        float a0, a1;
        f32x2_unpack(acc[k][p], a0, a1);
        const float l0 = round_act<T>(warp_sum_butterfly(a0));
        const float l1 = round_act<T>(warp_sum_butterfly(a1));
        if (lane == 0 && e < E) {
          const int t = 2 * p;
          ls[t * 64 + e] = l0;
          ls[(t + 1) * 64 + e] = l1;
          if (logits && t0 + t < tokens) logits[(t0 + t) * E + e] = from_f<T>(l0);
          if (logits && t0 + t + 1 < tokens) logits[(t0 + t + 1) * E + e] = from_f<T>(l1);
        }
      }
    }
  }
  __syncthreads();
  if (idx) {
    for (int t = warp; t < kRouterWideTokens && t0 + t < tokens; t += kRouterWideWarps) {
      const float la0 = lane < E ? ls[t * 64 + lane] : 0.f;
      const float la1 = lane + 32 < E ? ls[t * 64 + lane + 32] : 0.f;
      route_token<T>(lane, la0, la1, E, K, t0 + t, (T*)nullptr, idx, gates);
    }
  }
}

// Router for small batches (decode): a cluster of kRouterCluster CTAs per
// token, each computing ceil(E / kRouterCluster) experts (one warp per
// expert, the same fixed order as router_kernel), so the 64 dot products of
// a token run on 8 SMs at once instead of one after another on one.  Every
// CTA writes its act-rounded logits into CTA 0's shared memory (distributed
// shared memory); after the cluster barrier CTA 0's first warp ranks them.
constexpr int kRouterCluster = 8;

// The one-tile route sort (sort_one_tile_kernel's algorithm and output: a
// stable counting sort by expert) run by one 256-thread CTA over n <= 1024
// routes: route i = pass * 256 + thread is the 1024-thread kernel's thread i,
// so the per-warp counts, offsets and placement are the same.
constexpr int kFusedSortRoutes = 1024;
__device__ void sort_routes_cta(const int32_t* ids, int n, int E, const RouteSortOut& so) {
  __shared__ int32_t warp_cnt[kFusedSortRoutes / 32][64];
  __shared__ int32_t total[64];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int kPasses = kFusedSortRoutes / (kRouterBlockWarps * 32);
  for (int i = tid; i < (kFusedSortRoutes / 32) * E; i += blockDim.x) warp_cnt[i / E][i % E] = 0;
  __syncthreads();
  int ev[kPasses], rk[kPasses];
#pragma unroll
  for (int ps = 0; ps < kPasses; ++ps) {
    const int i = ps * kRouterBlockWarps * 32 + tid;
    const bool valid = i < n;
    const int e = valid ? __ldcg(&ids[i]) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (valid && rank == 0) warp_cnt[ps * kRouterBlockWarps + warp][e] = __popc(peers);
    ev[ps] = e;
    rk[ps] = rank;
  }
  __syncthreads();
  for (int x = tid; x < E; x += blockDim.x) {
    int32_t sum = 0;
    for (int w = 0; w < kFusedSortRoutes / 32; ++w) sum += warp_cnt[w][x];
    total[x] = sum;
  }
  __syncthreads();
  if (tid == 0) {
    int32_t run = 0, na = 0;
    for (int x = 0; x < E; ++x) {
      so.offsets[x] = run;
      const int32_t c = total[x];
      total[x] = run;
      run += c;
      if (c > 0) so.active[na++] = x;
    }
    so.offsets[E] = run;
    *so.active_count = na;
  }
  __syncthreads();
  for (int x = tid; x < E; x += blockDim.x) {
    int32_t run = total[x];
    for (int w = 0; w < kFusedSortRoutes / 32; ++w) {
      const int32_t c = warp_cnt[w][x];
      warp_cnt[w][x] = run;
      run += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int ps = 0; ps < kPasses; ++ps) {
    const int i = ps * kRouterBlockWarps * 32 + tid;
    if (i < n) {
      const int32_t pos = warp_cnt[ps * kRouterBlockWarps + warp][ev[ps]] + rk[ps];
      so.order[pos] = i;
      so.inverse[i] = pos;
    }
  }
}

template <typename T, bool DENSE, int J>
__global__ void __cluster_dims__(kRouterCluster, 1, 1) __launch_bounds__(kRouterBlockWarps * 32)
    router_cluster_kernel(const T* __restrict__ x, int64_t tokens, const T* __restrict__ wd,
                          const uint32_t* __restrict__ wq, const __half* __restrict__ ws,
                          const __half* __restrict__ wb, int E, int K, T* logits, int32_t* idx, T* gates,
                          const RouteSortOut so) {
  constexpr int H = J * 256;
  __shared__ float ls[64];
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int part = (int)cluster.block_rank();
  const int64_t t = blockIdx.x / kRouterCluster;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int epc = (E + kRouterCluster - 1) / kRouterCluster;  // experts per CTA (<= 8)
  const int e = part * epc + warp;
  if (warp < epc && e < E && t < tokens) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int c = lane + 32 * j;
      float xf[8], wf[8];
      unpack8<T>(ld_v4(x + t * H + 8 * c), xf);
      if (DENSE) {
        unpack8<T>(ld_v4(wd + (int64_t)e * H + 8 * c), wf);
      } else {
        const uint32_t word = wq[(int64_t)e * (H / 8) + c];
        const float sc = __half2float(ws[(int64_t)e * (H / 64) + c / 8]);
        const float bi = __half2float(wb[(int64_t)e * (H / 64) + c / 8]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float code = (float)((word >> (4 * i)) & 0xFu);
          wf[i] = __half2float(__float2half_rn(__fadd_rn(__fmul_rn(code, sc), bi)));
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) acc = __fadd_rn(acc, __fmul_rn(xf[i], wf[i]));
    }
    const float la = round_act<T>(warp_sum_butterfly(acc));
    if (lane == 0) {
      *cluster.map_shared_rank(&ls[e], 0) = la;
      if (logits) logits[t * E + e] = from_f<T>(la);
    }
  }
  cluster.sync();
  if (part == 0 && warp == 0 && idx && t < tokens) {
    const float la0 = lane < E ? ls[lane] : 0.f;
    const float la1 = lane + 32 < E ? ls[lane + 32] : 0.f;
    route_token<T>(lane, la0, la1, E, K, t, (T*)nullptr, idx, gates);
  }
  if (so.arrivals && part == 0) {
    // The last token's CTA to finish sorts every route (ids written by the
    // other clusters are read from L2 after the fences).
    __shared__ int last_s;
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      const int last = atomicAdd(so.arrivals, 1) == (int)tokens - 1;
      if (last) *so.arrivals = 0;  // left at zero for the next launch
      last_s = last;
    }
    __syncthreads();
    if (last_s) {
      __threadfence();
      sort_routes_cta(idx, (int)tokens * K, E, so);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kRouterWarps * 32)
    route_kernel(const T* __restrict__ logits, int64_t tokens, int E, int K, T* probs,
                 int32_t* idx, T* gates) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kRouterWarps + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const float la0 = lane < E ? to_f(logits[t * E + lane]) : 0.f;
  const float la1 = lane + 32 < E ? to_f(logits[t * E + lane + 32]) : 0.f;
  route_token<T>(lane, la0, la1, E, K, t, probs, idx, gates);
}

// Rank only (input already probabilities).
template <typename T>
__global__ void __launch_bounds__(kRouterWarps * 32)
    topk_kernel(const T* __restrict__ probs, int64_t rows, int E, int K, int32_t* idx) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kRouterWarps + (threadIdx.x >> 5);
  if (t >= rows) return;
  const float p0 = lane < E ? to_f(probs[t * E + lane]) : 0.f;
  const float p1 = lane + 32 < E ? to_f(probs[t * E + lane + 32]) : 0.f;
  const bool v0 = lane < E, v1 = lane + 32 < E;
  int r0 = 0, r1 = 0;
  const bool n0 = isnan(p0), n1 = isnan(p1);
  for (int j = 0; j < E; ++j) {
    const float o = __shfl_sync(0xffffffffu, j < 32 ? p0 : p1, j & 31);
    const bool on = isnan(o);
    r0 += ((!on && (n0 || o > p0)) || (((on && n0) || (!on && !n0 && o == p0)) && j < lane)) ? 1 : 0;
    r1 += ((!on && (n1 || o > p1)) || (((on && n1) || (!on && !n1 && o == p1)) && j < lane + 32)) ? 1 : 0;
  }
  if (v0 && r0 < K) idx[t * K + r0] = lane;
  if (v1 && r1 < K) idx[t * K + r1] = lane + 32;
}

template <typename T>
__global__ void take_along_kernel(const T* __restrict__ x, int64_t rows, int width,
                                  const int32_t* __restrict__ idx, int K, T* out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * K) return;
  const int64_t r = i / K;
  out[i] = x[r * width + idx[i]];
}

template <typename T, bool DENSE, int TPC>
static tf_status router_dispatch_tpc(const void* x, int64_t tokens, int hidden,
                                     const tf_router_weight& r, int E, int K, void* logits,
                                     int32_t* idx, void* gates, cudaStream_t s) {
  const unsigned blocks = (unsigned)((tokens + TPC - 1) / TPC);
  const T* wd = (const T*)r.dense;
  const uint32_t* wq = r.affine.q;
  const __half* wsc = (const __half*)r.affine.scales;
  const __half* wbi = (const __half*)r.affine.biases;
#define TF_ROUTER_CASE(JJ)                                                                  \
  case JJ:                                                                                  \
    router_kernel<T, DENSE, JJ, TPC><<<blocks, kRouterBlockWarps * 32, 0, s>>>(             \
        (const T*)x, tokens, wd, wq, wsc, wbi, E, K, (T*)logits, idx, (T*)gates);           \
    break;
  switch (hidden / 256) {
    TF_ROUTER_CASE(1)
    TF_ROUTER_CASE(2)
    TF_ROUTER_CASE(4)
    TF_ROUTER_CASE(8)
    default:
      return set_error(TF_ERR_UNSUPPORTED, "router: hidden %d not in {256,512,1024,2048}", hidden);
  }
#undef TF_ROUTER_CASE
  return check_launch("router");
}

template <typename T, bool DENSE, int J>
static tf_status router_wide_launch(const void* x, int64_t tokens, const tf_router_weight& r, int E, int K,
                                    void* logits, int32_t* idx, void* gates, cudaStream_t s) {
  constexpr size_t smem = router_wide_smem<J>();
  static PerDeviceOnce attr;
  int dev = 0;
  if (attr.needed(&dev)) {
    TF_CUDA(cudaFuncSetAttribute(router_wide_kernel<T, DENSE, J>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem));
    attr.mark(dev);
  }
  const unsigned blocks = (unsigned)((tokens + kRouterWideTokens - 1) / kRouterWideTokens);
  router_wide_kernel<T, DENSE, J><<<blocks, kRouterWideWarps * 32, smem, s>>>(
      (const T*)x, tokens, (const T*)r.dense, r.affine.q, (const __half*)r.affine.scales,
      (const __half*)r.affine.biases, E, K, (T*)logits, idx, (T*)gates);
  return check_launch("router_wide");
}

template <typename T, bool DENSE>
static tf_status router_dispatch_wide(const void* x, int64_t tokens, int hidden, const tf_router_weight& r,
                                      int E, int K, void* logits, int32_t* idx, void* gates, cudaStream_t s) {
  switch (hidden / 256) {
    case 1: return router_wide_launch<T, DENSE, 1>(x, tokens, r, E, K, logits, idx, gates, s);
    case 2: return router_wide_launch<T, DENSE, 2>(x, tokens, r, E, K, logits, idx, gates, s);
    case 4: return router_wide_launch<T, DENSE, 4>(x, tokens, r, E, K, logits, idx, gates, s);
    case 8: return router_wide_launch<T, DENSE, 8>(x, tokens, r, E, K, logits, idx, gates, s);
    default:
      return set_error(TF_ERR_UNSUPPORTED, "router: hidden %d not in {256,512,1024,2048}", hidden);
  }
}

template <typename T, bool DENSE>
static tf_status router_dispatch_cluster(const void* x, int64_t tokens, int hidden, const tf_router_weight& r,
                                         int E, int K, void* logits, int32_t* idx, void* gates, cudaStream_t s,
                                         const RouteSortOut& so) {
  const unsigned blocks = (unsigned)(tokens * kRouterCluster);
  const T* wd = (const T*)r.dense;
  const uint32_t* wq = r.affine.q;
  const __half* wsc = (const __half*)r.affine.scales;
  const __half* wbi = (const __half*)r.affine.biases;
#define TF_ROUTER_CCASE(JJ)                                                                  \
  case JJ:                                                                                   \
    router_cluster_kernel<T, DENSE, JJ><<<blocks, kRouterBlockWarps * 32, 0, s>>>(            \
        (const T*)x, tokens, wd, wq, wsc, wbi, E, K, (T*)logits, idx, (T*)gates, so);        \
    break;
  switch (hidden / 256) {
    TF_ROUTER_CCASE(1)
    TF_ROUTER_CCASE(2)
    TF_ROUTER_CCASE(4)
    TF_ROUTER_CCASE(8)
    default:
      return set_error(TF_ERR_UNSUPPORTED, "router: hidden %d not in {256,512,1024,2048}", hidden);
  }
#undef TF_ROUTER_CCASE
  return check_launch("router_cluster");
}

// Decode-sized batches: a cluster of 8 CTAs per token.  Up to 2048 tokens:
// one token per block; beyond, eight per block on packed fp32 pairs.
template <typename T, bool DENSE>
static tf_status router_dispatch(const void* x, int64_t tokens, int hidden,
                                 const tf_router_weight& r, int E, int K, void* logits,
                                 int32_t* idx, void* gates, cudaStream_t s, const RouteSortOut* sort,
                                 bool* sorted) {
  if (tokens <= 256) {
    // The route sort rides along when one CTA can take every route.
    RouteSortOut so;
    if (sort && sort->arrivals && idx && tokens * K <= kFusedSortRoutes && E <= 64) {
      so = *sort;
      if (sorted) *sorted = true;
    }
    return router_dispatch_cluster<T, DENSE>(x, tokens, hidden, r, E, K, logits, idx, gates, s, so);
  }
  if (tokens <= 2048)
    return router_dispatch_tpc<T, DENSE, 1>(x, tokens, hidden, r, E, K, logits, idx, gates, s);
  return router_dispatch_wide<T, DENSE>(x, tokens, hidden, r, E, K, logits, idx, gates, s);
}

tf_status launch_router(const void* x, int64_t tokens, int hidden, const tf_router_weight& r,
                        int E, int K, int act, void* logits, int32_t* idx, void* gates,
                        cudaStream_t s, const RouteSortOut* sort, bool* sorted) {
  if (sorted) *sorted = false;
  if (tokens == 0) return TF_OK;
  const bool dense = r.dense != nullptr;
  if (act == TF_DTYPE_F16)
    return dense ? router_dispatch<__half, true>(x, tokens, hidden, r, E, K, logits, idx, gates, s, sort, sorted)
                 : router_dispatch<__half, false>(x, tokens, hidden, r, E, K, logits, idx, gates, s, sort, sorted);
  return dense ? router_dispatch<__nv_bfloat16, true>(x, tokens, hidden, r, E, K, logits, idx, gates, s, sort,
                                                      sorted)
               : router_dispatch<__nv_bfloat16, false>(x, tokens, hidden, r, E, K, logits, idx, gates, s, sort,
                                                       sorted);
}

tf_status launch_route(const void* logits, int64_t tokens, int E, int K, int act, void* probs,
                       int32_t* idx, void* gates, cudaStream_t s) {
  if (tokens == 0) return TF_OK;
  const unsigned blocks = (unsigned)((tokens + kRouterWarps - 1) / kRouterWarps);
  if (act == TF_DTYPE_F16)
    route_kernel<__half><<<blocks, kRouterWarps * 32, 0, s>>>(
        (const __half*)logits, tokens, E, K, (__half*)probs, idx, (__half*)gates);
  else
    route_kernel<__nv_bfloat16><<<blocks, kRouterWarps * 32, 0, s>>>(
        (const __nv_bfloat16*)logits, tokens, E, K, (__nv_bfloat16*)probs, idx,
        (__nv_bfloat16*)gates);
  return check_launch("route");
}

tf_status launch_topk(const void* probs, int64_t rows, int E, int K, int act, int32_t* idx,
                      cudaStream_t s) {
  if (rows == 0) return TF_OK;
  const unsigned blocks = (unsigned)((rows + kRouterWarps - 1) / kRouterWarps);
  if (act == TF_DTYPE_F16)
    topk_kernel<__half><<<blocks, kRouterWarps * 32, 0, s>>>((const __half*)probs, rows, E, K, idx);
  else
    topk_kernel<__nv_bfloat16><<<blocks, kRouterWarps * 32, 0, s>>>((const __nv_bfloat16*)probs,
                                                                    rows, E, K, idx);
  return check_launch("topk");
}

tf_status launch_take_along(const void* x, int64_t rows, int width, const int32_t* idx, int K,
                            int act, void* out, cudaStream_t s) {
  const int64_t n = rows * K;
  if (n == 0) return TF_OK;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  if (act == TF_DTYPE_F16)
    take_along_kernel<__half><<<blocks, 256, 0, s>>>((const __half*)x, rows, width, idx, K,
                                                     (__half*)out);
  else
    take_along_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>((const __nv_bfloat16*)x, rows, width,
                                                            idx, K, (__nv_bfloat16*)out);
  return check_launch("take_along");
}

// ---------------------------------------------------------------------------
// Stable counting sort of expert ids.
//
// Tiles of kSortTile routes.  Pass 1 counts each tile's routes per expert;
// pass 2 (one block) turns the counts into global offsets, per-tile bases
// and the ascending list of active experts; pass 3 places every route at
// base[tile][e] + (routes of e earlier in the tile), using warp match masks
// plus a per-warp exclusive scan, so slot order equals flat order within an
// expert: order == stable argsort(ids).

constexpr int kSortTile = 1024;
constexpr int kSortMaxExperts = 256;

__global__ void __launch_bounds__(kSortTile)
    sort_count_kernel(const int32_t* __restrict__ ids, int64_t n, int E, int32_t* tile_counts) {
  __shared__ int32_t cnt[kSortMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  const int64_t i = (int64_t)blockIdx.x * kSortTile + threadIdx.x;
  if (i < n) atomicAdd(&cnt[ids[i]], 1);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) tile_counts[(int64_t)blockIdx.x * E + e] = cnt[e];
}

// One block of kSortMaxExperts threads; thread e owns expert e.
__global__ void __launch_bounds__(kSortMaxExperts)
    sort_scan_kernel(int64_t tiles, int E, int32_t* tile_counts, int32_t* offsets, int32_t* active,
                     int32_t* active_count) {
  __shared__ int32_t total[kSortMaxExperts];
  const int e = threadIdx.x;
  int32_t sum = 0;
  if (e < E)
    for (int64_t t = 0; t < tiles; ++t) sum += tile_counts[t * E + e];
  total[e] = e < E ? sum : 0;
  __syncthreads();
  if (e == 0) {
    int32_t run = 0, na = 0;
    for (int x = 0; x < E; ++x) {
      offsets[x] = run;
      const int32_t c = total[x];
      total[x] = run;
      run += c;
      if (c > 0) active[na++] = x;
    }
    offsets[E] = run;
    *active_count = na;
  }
  __syncthreads();
  if (e < E) {
    int32_t base = total[e];
    for (int64_t t = 0; t < tiles; ++t) {
      const int32_t c = tile_counts[t * E + e];
      tile_counts[t * E + e] = base;  // becomes the tile's base for expert e
      base += c;
    }
  }
}

__global__ void __launch_bounds__(kSortTile)
    sort_place_kernel(const int32_t* __restrict__ ids, int64_t n, int E,
                      const int32_t* __restrict__ tile_base, int32_t* order, int32_t* inverse) {
  __shared__ int32_t warp_cnt[kSortTile / 32][kSortMaxExperts];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (kSortTile / 32) * E; i += blockDim.x)
    warp_cnt[i / E][i % E] = 0;
  __syncthreads();
  const int64_t i = (int64_t)blockIdx.x * kSortTile + threadIdx.x;
  const bool valid = i < n;
  const int e = valid ? ids[i] : -1;
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (valid && rank == 0) warp_cnt[warp][e] = __popc(peers);
  __syncthreads();
  // Exclusive scan over warps per expert, seeded with the tile base.
  for (int x = threadIdx.x; x < E; x += blockDim.x) {
    int32_t run = tile_base[(int64_t)blockIdx.x * E + x];
    for (int w = 0; w < kSortTile / 32; ++w) {
      const int32_t c = warp_cnt[w][x];
      warp_cnt[w][x] = run;
      run += c;
    }
  }
  __syncthreads();
  if (valid) {
    const int32_t pos = warp_cnt[warp][e] + rank;
    order[pos] = (int32_t)i;
    inverse[i] = pos;
  }
}

// All of the above in one block when the routes fit one tile (decode
// batches): per-warp counts by match mask, per-expert totals, offsets and the
// active list, then the same placement.
__global__ void __launch_bounds__(kSortTile)
    sort_one_tile_kernel(const int32_t* __restrict__ ids, int n, int E, int32_t* order, int32_t* inverse,
                         int32_t* offsets, int32_t* active, int32_t* active_count) {
  __shared__ int32_t warp_cnt[kSortTile / 32][kSortMaxExperts];
  __shared__ int32_t total[kSortMaxExperts];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (kSortTile / 32) * E; i += blockDim.x) warp_cnt[i / E][i % E] = 0;
  __syncthreads();
  const int i = threadIdx.x;
  const bool valid = i < n;
  const int e = valid ? ids[i] : -1;
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const int rank = __popc(peers & ((1u << lane) - 1u));
  if (valid && rank == 0) warp_cnt[warp][e] = __popc(peers);
  __syncthreads();
  for (int x = threadIdx.x; x < E; x += blockDim.x) {
    int32_t sum = 0;
    for (int w = 0; w < kSortTile / 32; ++w) sum += warp_cnt[w][x];
    total[x] = sum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t run = 0, na = 0;
    for (int x = 0; x < E; ++x) {
      offsets[x] = run;
      const int32_t c = total[x];
      total[x] = run;
      run += c;
      if (c > 0) active[na++] = x;
    }
    offsets[E] = run;
    *active_count = na;
  }
  __syncthreads();
  for (int x = threadIdx.x; x < E; x += blockDim.x) {
    int32_t run = total[x];
    for (int w = 0; w < kSortTile / 32; ++w) {
      const int32_t c = warp_cnt[w][x];
      warp_cnt[w][x] = run;
      run += c;
    }
  }
  __syncthreads();
  if (valid) {
    const int32_t pos = warp_cnt[warp][e] + rank;
    order[pos] = i;
    inverse[i] = pos;
  }
}

__global__ void gather_index_kernel(const int32_t* __restrict__ src, const int32_t* __restrict__ perm,
                                    int64_t n, int div, int32_t* dst) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src ? src[perm[i]] / div : perm[i] / div;
}

size_t sort_workspace_bytes(int64_t n, int experts) {
  const int64_t tiles = (n + kSortTile - 1) / kSortTile;
  return align_up((size_t)(tiles > 0 ? tiles : 1) * experts * sizeof(int32_t), 256);
}

tf_status launch_route_sort(const int32_t* ids, int64_t n, int E, int32_t* order, int32_t* inverse,
                            int32_t* offsets, int32_t* active, int32_t* active_count, void* ws,
                            size_t ws_bytes, cudaStream_t s) {
  if (E > kSortMaxExperts)
    return set_error(TF_ERR_UNSUPPORTED, "route sort supports at most %d experts", kSortMaxExperts);
  if (ws_bytes < sort_workspace_bytes(n, E))
    return set_error(TF_ERR_INVALID_ARGUMENT, "route sort workspace too small");
  const int64_t tiles = (n + kSortTile - 1) / kSortTile;
  if (tiles == 1) {
    sort_one_tile_kernel<<<1, kSortTile, 0, s>>>(ids, (int)n, E, order, inverse, offsets, active, active_count);
    return check_launch("sort_one_tile");
  }
  int32_t* tile_counts = (int32_t*)ws;
  if (tiles > 0) {
    sort_count_kernel<<<(unsigned)tiles, kSortTile, 0, s>>>(ids, n, E, tile_counts);
    TF_TRY(check_launch("sort_count"));
  }
  sort_scan_kernel<<<1, kSortMaxExperts, 0, s>>>(tiles, E, tile_counts, offsets, active, active_count);
  TF_TRY(check_launch("sort_scan"));
  if (tiles > 0) {
    sort_place_kernel<<<(unsigned)tiles, kSortTile, 0, s>>>(ids, n, E, tile_counts, order, inverse);
    TF_TRY(check_launch("sort_place"));
  }
  return TF_OK;
}

tf_status launch_gather_index(const int32_t* src, const int32_t* perm, int64_t n, int div,
                              int32_t* dst, cudaStream_t s) {
  if (n == 0) return TF_OK;
  gather_index_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(src, perm, n, div, dst);
  return check_launch("gather_index");
}

}  // namespace tf
