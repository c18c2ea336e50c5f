// MLX-affine 4-bit QMM / gather_qmm as a memory-bound GEMV, whole rows per warp.
//
// Restates native_affine_gather_qmm / native_affine_qmm
// (overlays/executorch/backends/mlx/native_affine_ops.py:39-74) and the
// adapter's gather_qmm / quantized_matmul calls
// (MLXNativeGraniteMoEPrefill.h:539-550) for few tokens per weight matrix
// (decode).  y = act(sum_k x_k (code_k s_g + b_g)) with fp32 accumulation,
// evaluated per 32-element half-group as s_g * sum(x*code) + b_g * sum(x).
//
// Work is a list of (segment, block of 8 R output rows) items, grid-strided
// over a fixed grid so the launch never depends on device-side routing:
//   DENSE     - one segment (expert 0) holding every slot;
//   PER_ROUTE - slot n is its own segment with expert indices[n];
//   GROUPED   - active expert a owns slots offsets[e] .. offsets[e+1] (the
//               output of the route sort), so an expert's weights are read
//               once for all of its tokens.
// Each warp owns R rows, staged in shared memory by cp.async before use; lane
// l owns the 16-byte weight chunks l + 32m of a row (32 codes each) and keeps
// the matching activations in registers.
//
// Nibble decode: for code j (bits 4j) of a word w, j <= 4,
//   float(0x4B000000 | (w & (0xF << 4j))) - 2^23 == code_j * 16^j  (exact),
// so the activation is stored pre-multiplied by 16^-j (an exact power of two)
// and one LOP3 + one FADD + one FFMA handle a code.  Codes 5..7 use w >> 20.
#include "common.cuh"
#include "internal.h"

namespace tf {

constexpr int kGemvWarps = 8;

struct GemvArgs {
  const void* x;
  int64_t x_stride;
  const int32_t* x_index;
  int x_div;
  int rows_per_x;
  int64_t n;
  const int32_t* indices;
  const int32_t* offsets;
  const int32_t* active;
  const int32_t* active_count;
  const uint32_t* q0;
  const __half* s0;
  const __half* b0;
  const uint32_t* q1;
  const __half* s1;
  const __half* b1;
  int out;
  int in;
  int experts;
  void* y;
  int64_t y_stride;
  const int32_t* y_index;
  const void* residual;
  int64_t residual_stride;
};

__device__ __forceinline__ float nib(uint32_t masked) {
  return __int_as_float(0x4B000000u | masked) - 8388608.0f;
}

// Dot of one 32-code chunk (uint4) with pre-scaled activations xs[32].
__device__ __forceinline__ float chunk_dot(const uint4& wv, const float* xs) {
  const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
  float p = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t w = words[k];
    const uint32_t h = w >> 20;
    const float* xk = xs + 8 * k;
    p = fmaf(xk[0], nib(w & 0xFu), p);
    p = fmaf(xk[1], nib(w & 0xF0u), p);
    p = fmaf(xk[2], nib(w & 0xF00u), p);
    p = fmaf(xk[3], nib(w & 0xF000u), p);
    p = fmaf(xk[4], nib(w & 0xF0000u), p);
    p = fmaf(xk[5], nib(h & 0xFu), p);
    p = fmaf(xk[6], nib(h & 0xF0u), p);
    p = fmaf(xk[7], nib(h & 0xF00u), p);
  }
  return p;
}

// 16-byte global -> shared copy that bypasses L1 (weights are read once).
__device__ __forceinline__ void cp_async16(uint4* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

extern __shared__ __align__(16) uint4 gemv_smem[];

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

template <typename T, int MODE, int EPI, int TB, int M, int R>
__global__ void __launch_bounds__(kGemvWarps * 32) qmm_gemv_kernel(GemvArgs a) {
  constexpr int kGemvRows = kGemvWarps * R;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nrb = (a.out + kGemvRows - 1) / kGemvRows;
  const int nchunk = a.in / 32;
  int64_t nseg;
  if (MODE == QMM_DENSE) nseg = 1;
  else if (MODE == QMM_PER_ROUTE) nseg = a.n;
  else nseg = min(max(*a.active_count, 0), a.experts);
  const int64_t items = nseg * nrb;
  constexpr int NW = EPI == EPI_SWIGLU ? 2 : 1;
  // Pre-scale factors 16^-j for code position j of a word (j = i % 8).
  const float pre[8] = {1.f, 1.f / 16, 1.f / 256, 1.f / 4096, 1.f / 65536, 1.f, 1.f / 16, 1.f / 256};

  for (int64_t item = blockIdx.x; item < items; item += gridDim.x) {
    const int64_t seg = item / nrb;
    const int rb = (int)(item % nrb);
    int e;
    int64_t s0, s1;
    if (MODE == QMM_DENSE) {
      e = 0; s0 = 0; s1 = a.n;
    } else if (MODE == QMM_PER_ROUTE) {
      e = a.indices[seg]; s0 = seg; s1 = seg + 1;
    } else {
      // Clamped to [0, n] (see the tensor-core kernel's setup).
      e = min(max(a.active[seg], 0), a.experts - 1);
      s0 = min(max((int64_t)a.offsets[e], (int64_t)0), a.n);
      s1 = min(max((int64_t)a.offsets[e + 1], s0), a.n);
    }
    const int row0 = rb * kGemvRows + warp * R;
    // The weights of all R rows are requested before any is used, straight
    // into this warp's shared-memory slots (16-byte cp.async, no registers
    // held), together with their scales and biases, and before the
    // activations, so every round trip of the item overlaps: at one or a few
    // tokens the kernel is bound by bytes in flight, not by bandwidth. The
    // staged rows serve every slot of the segment. Each lane reads back only
    // the chunks it copied, so a per-thread wait suffices.
    uint4* wbuf = gemv_smem + (size_t)warp * (R * NW * M * 32) + lane;
    __half sr[R][NW][M], br[R][NW][M];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int row = row0 + r;
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const uint32_t* q = w == 0 ? a.q0 : a.q1;
        const __half* sc = w == 0 ? a.s0 : a.s1;
        const __half* bi = w == 0 ? a.b0 : a.b1;
        const int64_t wrow = (int64_t)e * a.out + row;
        const uint32_t* qrow = q + wrow * (a.in / 8);
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const int c = lane + 32 * m;
          const bool ok = row < a.out && c < nchunk;
          uint4* dst = wbuf + ((r * NW + w) * M + m) * 32;
          if (ok) cp_async16(dst, qrow + 4 * c);
          else *dst = make_uint4(0, 0, 0, 0);
          sr[r][w][m] = ok ? sc[wrow * (a.in / 64) + c / 2] : __float2half(0.f);
          br[r][w][m] = ok ? bi[wrow * (a.in / 64) + c / 2] : __float2half(0.f);
        }
      }
    }
    cp_async_commit();
    for (int64_t tb = s0; tb < s1; tb += TB) {
      // Activations of up to TB slots, pre-scaled, plus per-chunk sums.
      float xs[TB][M][32];
      float xsum[TB][M];
#pragma unroll
      for (int tt = 0; tt < TB; ++tt) {
        const int64_t slot = tb + tt;
#pragma unroll
        for (int m = 0; m < M; ++m) {
          xsum[tt][m] = 0.f;
          const int c = lane + 32 * m;
          if (slot < s1 && c < nchunk) {
            const int64_t xr = a.x_index ? a.x_index[slot] / a.x_div : slot / a.rows_per_x;
            const T* xp = (const T*)a.x + xr * a.x_stride + 32 * c;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              float f[8];
              unpack8<T>(ld_v4(xp + 8 * v), f);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                xsum[tt][m] += f[i];
                xs[tt][m][8 * v + i] = f[i] * pre[i];
              }
            }
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) xs[tt][m][i] = 0.f;
          }
        }
      }
      cp_async_wait_all();
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int row = row0 + r;
        if (row >= a.out) break;
        float acc[NW][TB];
#pragma unroll
        for (int w = 0; w < NW; ++w) {
#pragma unroll
          for (int tt = 0; tt < TB; ++tt) acc[w][tt] = 0.f;
#pragma unroll
          for (int m = 0; m < M; ++m) {
            const float s = __half2float(sr[r][w][m]);
            const float b = __half2float(br[r][w][m]);
            const uint4 wv = wbuf[((r * NW + w) * M + m) * 32];
#pragma unroll
            for (int tt = 0; tt < TB; ++tt)
              acc[w][tt] = fmaf(s, chunk_dot(wv, xs[tt][m]), fmaf(b, xsum[tt][m], acc[w][tt]));
          }
#pragma unroll
          for (int tt = 0; tt < TB; ++tt) acc[w][tt] = warp_sum_butterfly(acc[w][tt]);
        }
#pragma unroll
        for (int tt = 0; tt < TB; ++tt) {
          const int64_t slot = tb + tt;
          if (lane == tt && slot < s1) {
            T* yp = (T*)a.y + slot * a.y_stride + row;  // unused for EPI_F32
            if (EPI == EPI_SWIGLU) {
              const float g = round_act<T>(acc[0][tt]);
              const float u = round_act<T>(acc[NW - 1][tt]);
              *yp = from_f<T>(round_act<T>(silu_f(g)) * u);
            } else if (EPI == EPI_F32) {
              ((float*)a.y)[slot * a.y_stride + row] = round_act<T>(acc[0][tt]);
            } else if (EPI == EPI_RESIDUAL) {
              const float res = to_f(((const T*)a.residual)[slot * a.residual_stride + row]);
              *yp = from_f<T>(res + round_act<T>(acc[0][tt]));
            } else {
              const int64_t orow = a.y_index ? (int64_t)a.y_index[slot] : slot;
              ((T*)a.y)[orow * a.y_stride + row] = from_f<T>(acc[0][tt]);
            }
          }
        }
      }
    }
    // An empty segment skipped the wait above; its copies must land before
    // the next item reuses the slots.
    cp_async_wait_all();
  }
}

// Launch with R rows per warp. Each warp stages R x NW x M chunks of 512 bytes
// (4 KB, 32 KB per block); fewer rows per warp when that leaves under one
// block per SM, so a small matrix still spreads over every SM.
template <typename T, int MODE, int EPI, int TB, int M>
static tf_status gemv_launch(const GemvArgs& a, int64_t max_seg, cudaStream_t s) {
  constexpr int NW = EPI == EPI_SWIGLU ? 2 : 1;
  constexpr int RB = NW * M >= 8 ? 1 : 8 / (NW * M);
  constexpr int sms = 148;
  const int64_t nrb = (a.out + kGemvWarps * RB - 1) / (kGemvWarps * RB);
  const bool big = max_seg * nrb >= sms;
  const int rows = big ? RB : 1;
  const int64_t items = max_seg * ((a.out + kGemvWarps * rows - 1) / (kGemvWarps * rows));
  if (items <= 0) return TF_OK;
  const unsigned grid = (unsigned)(items < (int64_t)sms * 8 ? items : (int64_t)sms * 8);
  const size_t smem = (size_t)kGemvWarps * rows * NW * M * 32 * sizeof(uint4);
  if (big)
    qmm_gemv_kernel<T, MODE, EPI, TB, M, RB><<<grid, kGemvWarps * 32, smem, s>>>(a);
  else
    qmm_gemv_kernel<T, MODE, EPI, TB, M, 1><<<grid, kGemvWarps * 32, smem, s>>>(a);
  return check_launch("qmm_gemv");
}

template <typename T, int MODE, int EPI>
static tf_status qmm_dispatch(const GemvArgs& a, cudaStream_t s) {
  const int64_t max_seg = MODE == QMM_DENSE ? 1 : MODE == QMM_PER_ROUTE ? a.n : a.experts;
  if (a.in <= 1024) return gemv_launch<T, MODE, EPI, 2, 1>(a, max_seg, s);
  if (a.in <= 2048) return gemv_launch<T, MODE, EPI, 1, 2>(a, max_seg, s);
  return gemv_launch<T, MODE, EPI, 1, 4>(a, max_seg, s);
}

template <typename T>
static tf_status qmm_by_mode(const GemvArgs& a, int mode, int epi, cudaStream_t s) {
#define TF_QMM_EPI(MODE)                                                       \
  switch (epi) {                                                               \
    case EPI_PLAIN: return qmm_dispatch<T, MODE, EPI_PLAIN>(a, s);             \
    case EPI_SWIGLU: return qmm_dispatch<T, MODE, EPI_SWIGLU>(a, s);           \
    case EPI_F32: return qmm_dispatch<T, MODE, EPI_F32>(a, s);                 \
    default: return qmm_dispatch<T, MODE, EPI_RESIDUAL>(a, s);                 \
  }
  switch (mode) {
    case QMM_DENSE: TF_QMM_EPI(QMM_DENSE)
    case QMM_PER_ROUTE: TF_QMM_EPI(QMM_PER_ROUTE)
    default: TF_QMM_EPI(QMM_GROUPED)
  }
#undef TF_QMM_EPI
}

int g_qmm_path = 0;

bool qmm_uses_tc(const QmmProblem& p) {
  const int in = p.w0.in_features;
  const bool tc_ok = p.mode != QMM_PER_ROUTE && in % 512 == 0 && in <= 8192 &&
                     !(p.mode == QMM_DENSE && p.x_index);
  if (!tc_ok || g_qmm_path == 1) return false;
  if (g_qmm_path == 2) return true;
  if (p.mode == QMM_DENSE) return p.n >= 8;
  // The GEMV streams an expert's weights once per route, the tensor cores
  // once per expert.  Measured on B200 (OLMoE MoE block, 64 experts top-8):
  // 8 routes 70 (GEMV) vs 73 us (tensor cores), 16 routes 93 vs 82, 64
  // routes 197 vs 116, 128 routes 287 vs 135.
  return p.n >= 16;
}

tf_status launch_qmm(const QmmProblem& p, cudaStream_t s) {
  if (p.n == 0) return TF_OK;
  // The tensor cores read an f16 operand with contiguous rows: x itself for
  // dense f16, else the caller-provided copy.
  const bool operand = p.x16 || (p.mode == QMM_DENSE && p.act == TF_DTYPE_F16);
  if (qmm_uses_tc(p) && operand) return launch_qmm_tc(p, s);
  return launch_qmm_gemv(p, s);
}

tf_status launch_qmm_gemv(const QmmProblem& p, cudaStream_t s) {
  if (p.n == 0) return TF_OK;
  if (p.w0.in_features > 4096)
    return set_error(TF_ERR_UNSUPPORTED, "qmm: in_features %d > 4096", p.w0.in_features);
  GemvArgs a;
  a.x = p.x;
  a.x_stride = p.x_stride;
  a.x_index = p.x_index;
  a.x_div = p.x_div;
  a.rows_per_x = p.rows_per_x;
  a.n = p.n;
  a.indices = p.indices;
  a.offsets = p.offsets;
  a.active = p.active;
  a.active_count = p.active_count;
  a.q0 = p.w0.q;
  a.s0 = (const __half*)p.w0.scales;
  a.b0 = (const __half*)p.w0.biases;
  a.q1 = p.epilogue == EPI_SWIGLU ? p.w1.q : p.w0.q;
  a.s1 = (const __half*)(p.epilogue == EPI_SWIGLU ? p.w1.scales : p.w0.scales);
  a.b1 = (const __half*)(p.epilogue == EPI_SWIGLU ? p.w1.biases : p.w0.biases);
  a.out = p.w0.out_features;
  a.in = p.w0.in_features;
  a.experts = p.w0.experts > 0 ? p.w0.experts : 1;
  a.y = p.y;
  a.y_stride = p.y_stride;
  a.y_index = p.epilogue == EPI_PLAIN ? p.y_index : nullptr;
  a.residual = p.residual;
  a.residual_stride = p.residual_stride;
  if (p.act == TF_DTYPE_F16) return qmm_by_mode<__half>(a, p.mode, p.epilogue, s);
  return qmm_by_mode<__nv_bfloat16>(a, p.mode, p.epilogue, s);
}

}  // namespace tf
