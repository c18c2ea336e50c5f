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
//   append  (one block per row)   : norms, ropes, writes q (act) to scratch
//                                   and k/v (f16) into the cache slot pos[r];
//   split   (split, head, query)  : kSplit keys -> unnormalised (max, sum, o);
//   merge   (head, query)         : combines the splits in order.
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

// Sum of squares of a W-wide row in the canonical order (thread t owns the
// 8-element chunks t + 256 i; each 32 consecutive chunks form one butterfly
// group; group totals are added left to right).  Every thread gets the value.
template <typename T>
__device__ float block_row_sumsq(const T* row, int W, float* tot_s, float* bcast) {
  const int t = threadIdx.x, lane = t & 31;
  for (int c = t; 8 * c < W; c += kAttnThreads) {
    float f[8];
    unpack8<T>(ld_v4(row + 8 * c), f);
    const float v = warp_sum_butterfly(chunk_sumsq8(f));
    if (lane == 0) tot_s[c / 32] = v;
  }
  __syncthreads();
  if (t == 0) {
    float tot = tot_s[0];
    for (int i = 1; i < W / 256; ++i) tot = __fadd_rn(tot, tot_s[i]);
    *bcast = tot;
  }
  __syncthreads();
  const float v = *bcast;
  __syncthreads();
  return v;
}

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

template <typename T>
__global__ void __launch_bounds__(kAttnThreads)
    attn_append_kernel(const T* __restrict__ qkv, int heads, const __half* __restrict__ qn,
                       const __half* __restrict__ kn, float eps, float theta,
                       const int32_t* __restrict__ pos, const int32_t* __restrict__ req,
                       __half* k_cache, __half* v_cache, int cap, T* __restrict__ q_out,
                       const float2* __restrict__ rope) {
  __shared__ float tot_s[64];
  __shared__ float bcast;
  __shared__ float inv_s[kHeadDim / 2];  // RoPE inverse frequencies theta^(-2d/D)
  const int64_t r = blockIdx.x;
  const int t = threadIdx.x;
  const int W = heads * kHeadDim;
  if (!rope)
    for (int d = t; d < kHeadDim / 2; d += kAttnThreads)
      inv_s[d] = (float)pow((double)theta, -2.0 * (double)d / (double)kHeadDim);  // (synced below)
  const T* qrow = qkv + r * 3 * W;
  const T* krow = qrow + W;
  const T* vrow = qrow + 2 * W;
  const int p = pos[r];
  const int64_t q_req = req ? req[r] : r;
  const float rq = rms_scale(block_row_sumsq<T>(qrow, W, tot_s, &bcast), W, eps);
  const float rk = rms_scale(block_row_sumsq<T>(krow, W, tot_s, &bcast), W, eps);
  const float fp = (float)p;
  for (int i = t; i < W / 2; i += kAttnThreads) {
    const int h = i / (kHeadDim / 2), d = i % (kHeadDim / 2);
    const int i1 = h * kHeadDim + d, i2 = i1 + kHeadDim / 2;
    float sn, cs;
    if (rope) {
      const float2 a = rope[(int64_t)p * (kHeadDim / 2) + d];
      cs = a.x, sn = a.y;
    } else {
      sincosf(__fmul_rn(fp, inv_s[d]), &sn, &cs);
    }
    {
      const float x1 = round_act<T>(__fmul_rn(__fmul_rn(to_f(qrow[i1]), rq), __half2float(qn[i1])));
      const float x2 = round_act<T>(__fmul_rn(__fmul_rn(to_f(qrow[i2]), rq), __half2float(qn[i2])));
      q_out[r * W + i1] = from_f<T>(x1 * cs - x2 * sn);
      q_out[r * W + i2] = from_f<T>(x1 * sn + x2 * cs);
    }
    {
      const float x1 = round_act<T>(__fmul_rn(__fmul_rn(to_f(krow[i1]), rk), __half2float(kn[i1])));
      const float x2 = round_act<T>(__fmul_rn(__fmul_rn(to_f(krow[i2]), rk), __half2float(kn[i2])));
      const int64_t slot = ((q_req * heads + h) * cap + p) * kHeadDim;
      k_cache[slot + d] = __float2half_rn(round_act<T>(x1 * cs - x2 * sn));
      k_cache[slot + d + kHeadDim / 2] = __float2half_rn(round_act<T>(x1 * sn + x2 * cs));
    }
  }
  for (int i = t; i < W; i += kAttnThreads) {
    const int h = i / kHeadDim, d = i % kHeadDim;
    v_cache[((q_req * heads + h) * cap + p) * kHeadDim + d] = __float2half_rn(to_f(vrow[i]));
  }
}

template <typename T>
__global__ void __launch_bounds__(kAttnThreads)
    attn_split_kernel(const T* __restrict__ q, int heads, const int32_t* __restrict__ pos,
                      const int32_t* __restrict__ req, const int32_t* __restrict__ qrows,
                      const __half* __restrict__ k_cache, const __half* __restrict__ v_cache, int cap,
                      float scale, int nsplit, float* __restrict__ pm, float* __restrict__ pl,
                      float* __restrict__ po) {
  __shared__ float sc[kSplit];
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
}

template <typename T>
__global__ void __launch_bounds__(kHeadDim)
    attn_merge_kernel(const int32_t* __restrict__ pos, const int32_t* __restrict__ qrows, int heads, int nsplit,
                      const float* __restrict__ pm, const float* __restrict__ pl,
                      const float* __restrict__ po, T* __restrict__ out) {
  const int h = blockIdx.x, d = threadIdx.x;
  const int64_t z = blockIdx.y;
  const int64_t r = qrows ? qrows[z] : z;
  const int L = pos[r] + 1;
  const int ns = (L + kSplit - 1) / kSplit;
  const int64_t base = (z * heads + h) * nsplit;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, pm[base + s]);
  float acc = 0.f, l = 0.f;
  for (int s = 0; s < ns; ++s) {
    const float w = expf(pm[base + s] - M);
    acc = fmaf(w, po[(base + s) * kHeadDim + d], acc);
    l = fmaf(w, pl[base + s], l);
  }
  out[z * heads * kHeadDim + h * kHeadDim + d] = from_f<T>(acc / l);
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
  T* qr = c.take<T>((size_t)a.rows * a.heads * kHeadDim * sizeof(T));
  float* pm = c.take<float>(parts * 4);
  float* pl = c.take<float>(parts * 4);
  float* po = c.take<float>(parts * kHeadDim * 4);
  attn_append_kernel<T><<<(unsigned)a.rows, kAttnThreads, 0, s>>>(
      (const T*)a.qkv, a.heads, (const __half*)a.q_norm, (const __half*)a.k_norm, a.eps, a.theta,
      a.pos, a.req, (__half*)a.k_cache, (__half*)a.v_cache, a.capacity, qr, (const float2*)a.rope);
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
                                                     nsplit, pm, pl, po);
  TF_TRY(check_launch("attn_split"));
  dim3 mgrid(a.heads, (unsigned)nq);
  attn_merge_kernel<T><<<mgrid, kHeadDim, 0, s>>>(a.pos, a.qrows, a.heads, nsplit, pm, pl, po, (T*)a.out);
  return check_launch("attn_merge");
}

tf_status launch_attention(const AttnProblem& a, cudaStream_t s) {
  if (a.rows == 0) return TF_OK;
  if (a.head_dim != kHeadDim)
    return set_error(TF_ERR_UNSUPPORTED, "attention: head_dim %d (only %d)", a.head_dim, kHeadDim);
  const int W = a.heads * kHeadDim;
  if (W % 256 != 0 || W > 256 * 64)
    return set_error(TF_ERR_UNSUPPORTED, "attention: width %d", W);
  if (a.ws_bytes < attention_ws_bytes(a.rows, a.heads, a.capacity, a.act))
    return set_error(TF_ERR_INVALID_ARGUMENT, "attention workspace too small");
  if (a.max_len < 1 || a.max_len > a.capacity)
    return set_error(TF_ERR_CAPACITY, "attention: length %d outside [1, %d]", a.max_len, a.capacity);
  if (a.act == TF_DTYPE_F16) return attention_impl<__half>(a, s);
  return attention_impl<__nv_bfloat16>(a, s);
}

}  // namespace tf
