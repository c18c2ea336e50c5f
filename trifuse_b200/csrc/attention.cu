// fp16 KV-cache attention with full-width Q/K RMSNorm, RoPE and KV append.
//
// Restates the attention of NativeGraniteMoEPrefill::run
// (MLXNativeGraniteMoEPrefill.h:448-483):
//   q/k = rms_norm over the full projection width, before the head split
//         (448-453); RoPE half-split with base theta at each row's absolute
//         position (457-458); k/v appended to the fp16 cache
//         (MLXSequenceCache::update_and_fetch, patches/executorch.patch:
//         3357-3405); SDPA with scale 1/sqrt(D), causal for T > 1 (474-482).
//
// A "row" is one query token: row r belongs to request req[r] (identity when
// req is NULL) and sits at absolute position pos[r]; it attends the slots
// 0..pos[r] of its request's cache, which is exactly the causal mask for a
// prefill chunk and the full history for decode.
//
//   append  (one warp per row)    : norms, ropes, writes q (act) to scratch
//                                   and k/v (f16) into the cache slot pos[r];
//   split   (split, head, query)  : kSplit keys -> unnormalised (max, sum, o);
//                                   the last split block of a (head, query)
//                                   to finish combines the splits in order.
// Prefill rows grouped per request run the tensor-core kernel (attn_tc.cu)
// after the append instead of split.
// The queries are every row, or a listed subset (the last row of each
// request in the last layer of a prefill, MLXNativeGraniteMoEPrefill.h:
// 440-442, 471), or none (a cache-only chunk's last layer, :470).
// K/V rows stream with 128-bit loads, a half-warp per 256-byte key row.
#include <math.h>

#include "common.cuh"
#include "internal.h"

namespace tf {

constexpr int kHeadDim = 128;
constexpr int kSplit = 256;
constexpr int kAttnThreads = 256;
constexpr int kKeyGroups = kAttnThreads / 16;  // half-warps per block

// RoPE angles of every position below `positions`: tab[p][d] = (cos, sin)
// of fp32(p * theta^(-2d/D)), the values the append kernel computes.
__global__ void rope_table_kernel(float theta, int positions, float2* __restrict__ tab) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)positions * (kHeadDim / 2)) return;
  const int p = (int)(i / (kHeadDim / 2)), d = (int)(i % (kHeadDim / 2));
  const float inv = (float)pow((double)theta, -2.0 * (double)d / (double)kHeadDim);
  float sn, cs;
  sincosf(__fmul_rn((float)p, inv), &sn, &cs);
  tab[i] = make_float2(cs, sn);
}

// One warp per row (8 rows per block, no block barriers): Q/K RMSNorm,
// RoPE, K/V append.  Lane l holds the 8-element chunks c = l + 32 m of a
// row, so group m of 32 chunks is one warp butterfly, and the group totals
// add in m order: the sum of squares is rms_norm_kernel's order (chunk sums,
// butterflies over 32 chunks, group totals in order), bit-identical.  A
// chunk's RoPE partner (the same head's other half, chunk c + 8) sits in
// lane l ^ 8.  The row's width is W = heads * 128 <= 256 * 64.
constexpr int kAppendRows = 8;

template <typename T>
__device__ __forceinline__ float warp_row_sumsq(const T* row, int groups, int lane, float (*f)[8]) {
  float tot = 0.f;
  for (int m = 0; m < groups; ++m) {
    const float v = warp_sum_butterfly(chunk_sumsq8(f[m]));
    tot = m == 0 ? v : __fadd_rn(tot, v);
  }
  return tot;
}

template <typename T, int G>
__global__ void __launch_bounds__(kAppendRows * 32)
    attn_append_kernel(const T* __restrict__ qkv, int64_t rows, int heads, const __half* __restrict__ qn,
                       const __half* __restrict__ kn, float eps, float theta, const int32_t* __restrict__ pos,
                       const int32_t* __restrict__ req, __half* k_cache, __half* v_cache, int cap,
                       T* __restrict__ q_out, const float2* __restrict__ rope) {
  __shared__ float inv_s[kHeadDim / 2];  // RoPE inverse frequencies theta^(-2d/D) (no table)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (!rope) {
    for (int d = threadIdx.x; d < kHeadDim / 2; d += blockDim.x)
      inv_s[d] = (float)pow((double)theta, -2.0 * (double)d / (double)kHeadDim);
    __syncthreads();
  }
  const int64_t r = (int64_t)blockIdx.x * kAppendRows + warp;
  if (r >= rows) return;
  const int W = heads * kHeadDim;
  const T* qrow = qkv + r * 3 * W;
  const T* krow = qrow + W;
  const T* vrow = qrow + 2 * W;
  const int p = pos[r];
  const int64_t q_req = req ? req[r] : r;
  const int64_t kv_row = (q_req * heads) * cap + p;  // cache row of head 0 at this position
  const bool first = (lane & 8) == 0;                // this lane's chunks are a head's first half
  const int dh = (lane & 7) * 8;                     // rotation index of the chunk's element 0
  float cs[8], sn[8];
  if (rope) {
    const float4* rp = reinterpret_cast<const float4*>(rope + (int64_t)p * (kHeadDim / 2) + dh);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 a = rp[k];
      cs[2 * k] = a.x, sn[2 * k] = a.y, cs[2 * k + 1] = a.z, sn[2 * k + 1] = a.w;
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) sincosf(__fmul_rn((float)p, inv_s[dh + k]), &sn[k], &cs[k]);
  }
  float f[G][8];
  // q: norm, rotate, store
#pragma unroll
  for (int m = 0; m < G; ++m) unpack8<T>(ld_v4(qrow + 8 * (lane + 32 * m)), f[m]);
  const float rq = rms_scale(warp_row_sumsq<T>(qrow, G, lane, f), W, eps);
#pragma unroll
  for (int m = 0; m < G; ++m) {
    const int c = lane + 32 * m;
    float w[8], x[8], o[8];
    unpack8<__half>(ld_v4(qn + 8 * c), w);
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] = round_act<T>(__fmul_rn(__fmul_rn(f[m][k], rq), w[k]));
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float y = __shfl_xor_sync(0xffffffffu, x[k], 8);  // the partner half
      const float x1 = first ? x[k] : y, x2 = first ? y : x[k];
      o[k] = first ? x1 * cs[k] - x2 * sn[k] : x1 * sn[k] + x2 * cs[k];
    }
    *reinterpret_cast<uint4*>(q_out + r * W + 8 * c) = pack8<T>(o);
  }
  // k: norm, rotate, append
#pragma unroll
  for (int m = 0; m < G; ++m) unpack8<T>(ld_v4(krow + 8 * (lane + 32 * m)), f[m]);
  const float rk = rms_scale(warp_row_sumsq<T>(krow, G, lane, f), W, eps);
#pragma unroll
  for (int m = 0; m < G; ++m) {
    const int c = lane + 32 * m;
    float w[8], x[8], o[8];
    unpack8<__half>(ld_v4(kn + 8 * c), w);
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] = round_act<T>(__fmul_rn(__fmul_rn(f[m][k], rk), w[k]));
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float y = __shfl_xor_sync(0xffffffffu, x[k], 8);
      const float x1 = first ? x[k] : y, x2 = first ? y : x[k];
      o[k] = round_act<T>(first ? x1 * cs[k] - x2 * sn[k] : x1 * sn[k] + x2 * cs[k]);
    }
    const int h = c / (kHeadDim / 8), d0 = (c % (kHeadDim / 8)) * 8;
    *reinterpret_cast<uint4*>(k_cache + (kv_row + (int64_t)h * cap) * kHeadDim + d0) = pack8<__half>(o);
  }
  // v: append
#pragma unroll
  for (int m = 0; m < G; ++m) {
    const int c = lane + 32 * m;
    float v[8];
    unpack8<T>(ld_v4(vrow + 8 * c), v);
    const int h = c / (kHeadDim / 8), d0 = (c % (kHeadDim / 8)) * 8;
    *reinterpret_cast<uint4*>(v_cache + (kv_row + (int64_t)h * cap) * kHeadDim + d0) = pack8<__half>(v);
  }
}

// The split blocks of one (query, head) count their arrivals; the last one
// to arrive merges every part (in split order, as a separate merge launch
// would) and leaves the counter at zero, so no separate merge launch
// waits behind the slowest split.
template <typename T>
__device__ __forceinline__ void attn_merge_last(const int32_t* __restrict__ pos, int64_t r, int64_t z, int h,
                                                int heads, int nsplit, const float* pm, const float* pl,
                                                const float* po, int* arrivals, T* __restrict__ out, int* last_s) {
  __syncthreads();  // this block's part is written
  if (threadIdx.x == 0) {
    __threadfence();
    int* ctr = &arrivals[z * heads + h];
    const int seen = atomicAdd(ctr, 1);
    const int last = seen == (int)gridDim.x - 1;
    if (last) *ctr = 0;  // left at zero for the next launch
    *last_s = last;
  }
  __syncthreads();
  if (!*last_s) return;
  __threadfence();
  const int d = threadIdx.x;
  if (d >= kHeadDim) return;
  const int L = pos[r] + 1;
  const int ns = (L + kSplit - 1) / kSplit;
  const int64_t base = (z * heads + h) * nsplit;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, __ldcg(&pm[base + s]));
  float acc = 0.f, l = 0.f;
  for (int s = 0; s < ns; ++s) {
    const float w = expf(__ldcg(&pm[base + s]) - M);
    acc = fmaf(w, __ldcg(&po[(base + s) * kHeadDim + d]), acc);
    l = fmaf(w, __ldcg(&pl[base + s]), l);
  }
  out[z * heads * kHeadDim + h * kHeadDim + d] = from_f<T>(acc / l);
}

template <typename T>
__global__ void __launch_bounds__(kAttnThreads)
    attn_split_kernel(const T* __restrict__ q, int heads, const int32_t* __restrict__ pos,
                      const int32_t* __restrict__ req, const int32_t* __restrict__ qrows,
                      const __half* __restrict__ k_cache, const __half* __restrict__ v_cache, int cap,
                      float scale, int nsplit, float* __restrict__ pm, float* __restrict__ pl,
                      float* __restrict__ po, int* __restrict__ arrivals, T* __restrict__ out) {
  __shared__ float sc[kSplit];
  __shared__ int last_s;
  __shared__ float red[kAttnThreads / 32];
  __shared__ float opart[kKeyGroups][kHeadDim];
  const int s = blockIdx.x, h = blockIdx.y;
  const int64_t z = blockIdx.z;                  // output (query) index
  const int64_t r = qrows ? qrows[z] : z;        // its row among the appended rows
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int L = pos[r] + 1;
  const int k0 = s * kSplit;
  const int64_t part = (z * heads + h) * nsplit + s;
  if (k0 >= L) {
    if (t == 0) {
      pm[part] = -INFINITY;
      pl[part] = 0.f;
    }
    attn_merge_last<T>(pos, r, z, h, heads, nsplit, pm, pl, po, arrivals, out, &last_s);
    return;
  }
  const int k1 = min(L, k0 + kSplit);
  const int64_t head_base = ((req ? (int64_t)req[r] : r) * heads + h) * cap;
  // Half-warp g = 2*warp + half handles keys k0 + g + 16 i; lane dl holds dims
  // 8dl..8dl+7.  Loop bounds are warp-uniform (shuffles inside).
  const int half = (t >> 4) & 1, g = t >> 4, dl = t & 15;
  float qr[8];
  unpack8<T>(ld_v4(q + r * heads * kHeadDim + h * kHeadDim + 8 * dl), qr);
  const __half* kbase = k_cache + head_base * kHeadDim + 8 * dl;
  float mloc = -INFINITY;
  constexpr int U = 4;
  for (int jb = k0 + 2 * warp; jb < k1; jb += kKeyGroups * U) {
    uint4 kv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = jb + half + u * kKeyGroups;
      kv[u] = j < k1 ? ld_stream_v4(kbase + (int64_t)j * kHeadDim) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = jb + half + u * kKeyGroups;
      const __half2* kh = reinterpret_cast<const __half2*>(&kv[u]);
      float d = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 kf = __half22float2(kh[i]);
        d = fmaf(qr[2 * i], kf.x, d);
        d = fmaf(qr[2 * i + 1], kf.y, d);
      }
      d += __shfl_xor_sync(0xffffffffu, d, 8);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      if (j < k1) {
        const float sv = d * scale;
        mloc = fmaxf(mloc, sv);
        if (dl == 0) sc[j - k0] = sv;
      }
    }
  }
  mloc = warp_max(mloc);
  if (lane == 0) red[warp] = mloc;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int i = 1; i < kAttnThreads / 32; ++i) m = fmaxf(m, red[i]);
  __syncthreads();
  float lsum = 0.f;
  for (int j = t; j < k1 - k0; j += kAttnThreads) {
    const float p = expf(sc[j] - m);
    sc[j] = p;
    lsum += p;
  }
  lsum = warp_sum_butterfly(lsum);
  if (lane == 0) red[warp] = lsum;
  __syncthreads();
  float o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.f;
  const __half* vbase = v_cache + head_base * kHeadDim + 8 * dl;
  for (int jb = k0 + 2 * warp; jb < k1; jb += kKeyGroups * U) {
    uint4 vv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = jb + half + u * kKeyGroups;
      vv[u] = j < k1 ? ld_stream_v4(vbase + (int64_t)j * kHeadDim) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = jb + half + u * kKeyGroups;
      if (j < k1) {
        const float p = sc[j - k0];
        const __half2* vh = reinterpret_cast<const __half2*>(&vv[u]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 vf = __half22float2(vh[i]);
          o[2 * i] = fmaf(p, vf.x, o[2 * i]);
          o[2 * i + 1] = fmaf(p, vf.y, o[2 * i + 1]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) opart[g][8 * dl + i] = o[i];
  __syncthreads();
  if (t < kHeadDim) {
    float acc = 0.f;
#pragma unroll
    for (int gg = 0; gg < kKeyGroups; ++gg) acc += opart[gg][t];
    po[part * kHeadDim + t] = acc;
  }
  if (t == 0) {
    float l = 0.f;
    for (int i = 0; i < kAttnThreads / 32; ++i) l += red[i];
    pm[part] = m;
    pl[part] = l;
  }
  attn_merge_last<T>(pos, r, z, h, heads, nsplit, pm, pl, po, arrivals, out, &last_s);
}

// ---------------------------------------------------------------------------
tf_status launch_rope_table(float theta, int positions, void* tab, cudaStream_t s) {
  const int64_t n = (int64_t)positions * (kHeadDim / 2);
  if (n == 0) return TF_OK;
  rope_table_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(theta, positions, (float2*)tab);
  return check_launch("rope_table");
}

size_t attention_ws_bytes(int64_t rows, int heads, int capacity, int act) {
  const int64_t nsplit = (capacity + kSplit - 1) / kSplit;
  const int64_t parts = rows * heads * nsplit;
  Carve c(nullptr, 0);
  c.take<int>((size_t)rows * heads * 4);  // split arrivals first (zero between launches)
  c.take<char>((size_t)rows * heads * kHeadDim * act_bytes(act));  // roped q
  c.take<float>(parts * 4);
  c.take<float>(parts * 4);
  c.take<float>(parts * kHeadDim * 4);
  return c.used;
}

template <typename T>
static tf_status attention_impl(const AttnProblem& a, cudaStream_t s) {
  const int nsplit = (a.capacity + kSplit - 1) / kSplit;
  const int grid_splits = (a.max_len + kSplit - 1) / kSplit;
  const int64_t parts = a.rows * a.heads * nsplit;
  Carve c(a.ws, a.ws_bytes);
  // The arrival counters sit at the start, sized for the rows the workspace
  // was made for, so every call finds the same zeroed counters.
  const int64_t ws_rows = a.ws_rows > a.rows ? a.ws_rows : a.rows;
  int* arrivals = c.take<int>((size_t)ws_rows * a.heads * 4);
  T* qr = c.take<T>((size_t)a.rows * a.heads * kHeadDim * sizeof(T));
  float* pm = c.take<float>(parts * 4);
  float* pl = c.take<float>(parts * 4);
  float* po = c.take<float>(parts * kHeadDim * 4);
  if (!a.arrivals_zero) TF_CUDA(cudaMemsetAsync(arrivals, 0, (size_t)a.rows * a.heads * 4, s));
  {
    const unsigned blocks = (unsigned)((a.rows + kAppendRows - 1) / kAppendRows);
#define TF_APPEND(GG)                                                                                        \
  attn_append_kernel<T, GG><<<blocks, kAppendRows * 32, 0, s>>>(                                            \
      (const T*)a.qkv, a.rows, a.heads, (const __half*)a.q_norm, (const __half*)a.k_norm, a.eps, a.theta,   \
      a.pos, a.req, (__half*)a.k_cache, (__half*)a.v_cache, a.capacity, qr, (const float2*)a.rope)
    switch (a.heads * kHeadDim / 256) {
      case 1: TF_APPEND(1); break;
      case 2: TF_APPEND(2); break;
      case 4: TF_APPEND(4); break;
      case 8: TF_APPEND(8); break;
      case 16: TF_APPEND(16); break;
      default: return set_error(TF_ERR_UNSUPPORTED, "attention: width %d", a.heads * kHeadDim);
    }
#undef TF_APPEND
  }
  TF_TRY(check_launch("attn_append"));
  // Queries: every row, or only the rows a.qrows lists (output row i for
  // a.qrows[i]); none when a.nq == 0 (the rows only extend the cache).
  const int64_t nq = a.qrows ? a.nq : a.rows;
  if (nq == 0) return TF_OK;
  if (a.qblocks && a.nqblocks > 0 && !a.qrows) {
    // Prefill rows grouped per request: tiled tensor-core attention.
    return launch_attn_prefill_tc(a, qr, s);
  }
  dim3 grid(grid_splits, a.heads, (unsigned)nq);
  attn_split_kernel<T><<<grid, kAttnThreads, 0, s>>>(qr, a.heads, a.pos, a.req, a.qrows,
                                                     (const __half*)a.k_cache,
                                                     (const __half*)a.v_cache, a.capacity, a.scale,
                                                     nsplit, pm, pl, po, arrivals, (T*)a.out);
  return check_launch("attn_split");
}

tf_status launch_attention(const AttnProblem& a, cudaStream_t s) {
  if (a.rows == 0) return TF_OK;
  if (a.head_dim != kHeadDim)
    return set_error(TF_ERR_UNSUPPORTED, "attention: head_dim %d (only %d)", a.head_dim, kHeadDim);
  const int W = a.heads * kHeadDim;
  if (W % 256 != 0 || W > 256 * 64)
    return set_error(TF_ERR_UNSUPPORTED, "attention: width %d", W);
  if (a.ws_bytes < attention_ws_bytes(a.ws_rows > a.rows ? a.ws_rows : a.rows, a.heads, a.capacity, a.act))
    return set_error(TF_ERR_INVALID_ARGUMENT, "attention workspace too small");
  if (a.max_len < 1 || a.max_len > a.capacity)
    return set_error(TF_ERR_CAPACITY, "attention: length %d outside [1, %d]", a.max_len, a.capacity);
  if (a.act == TF_DTYPE_F16) return attention_impl<__half>(a, s);
  return attention_impl<__nv_bfloat16>(a, s);
}

}  // namespace tf
