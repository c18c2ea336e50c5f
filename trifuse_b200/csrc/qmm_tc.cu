// MLX-affine 4-bit grouped QMM on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), for many tokens per weight matrix (batched decode
// and prefill).
//
// Restates native_affine_gather_qmm / quantized_matmul
// (overlays/executorch/backends/mlx/native_affine_ops.py:39-74,
// MLXNativeGraniteMoEPrefill.h:539-550, 685-687) as D = W_e . X^T per expert:
// weight rows are the MMA's M side (128 per tile) and the expert's tokens the
// N side (NT per tile, N = tokens rounded up to 16), so a tile with few
// tokens still fills the 128-row MMA.  The MMA runs f16 x f16 -> f32: the
// weights are dequantized to fp16(code*s + b), the dtype the reference
// rounds its dequantized weight to (its float16 scale dtype,
// native_affine_ops.py:36); activations arrive in f16 (bf16 models pass an
// exact f16 copy).
//
// Persistent, warp-specialized blocks.  Work moves in stages of KS k-steps
// (a k-step is 64 inputs = one quantization group).  A block has G dequant
// groups of 8 warps, then 4 epilogue warps, the code loader, the MMA warp and
// the activation loader (Roles<G>):
//   dequant   groups take alternate stages.  In a group one thread per A row
//             and half k-step (warp w owns TMEM lanes 32(w%4).. and k half
//             (w/4)%2) turns packed words into f16 weights (magic-number half2
//             extraction + HFMA2) and writes them with tcgen05.st straight
//             into tensor memory: the A operand of each stage lives in TMEM
//             (row = lane, two k per 32-bit column).
//   epilogue  tcgen05.ld the finished accumulator while the next tile
//             accumulates into the other one; SwiGLU tiles keep gate row j
//             and up row j in adjacent TMEM lanes and the two lanes of a pair
//             each finish half of the tokens.
//   code loader  TMA of each stage's packed codes (box 8*KS words x 128 rows)
//             into a PK-deep ring, and of the scales and biases of every 8
//             k-steps (box 8 x 128) into two slots.
//   MMA       allocates the block's TMEM columns (two NT-column accumulators,
//             then SA stages of A); one elected lane issues tcgen05.mma with A
//             from TMEM and B from shared memory (4 x K=16 per k-step), waits
//             once on the A stage and once on the B stage, and commits each
//             stage to both release barriers.
//   activation loader  TMA of each stage's activation tiles (box 64 x NT,
//             128B-swizzled = the MMA's K-major layout) into an SB-deep ring.
// G = 1 (decode expert tiles): two blocks per SM with 256 TMEM columns each,
// so two MMA issuers run side by side (a small-N MMA is issue-bound).  G = 2
// (dense decode projections, prefill): one block per SM with all 512.
// Keeping A out of shared memory matters: a dequantized k-step is 16 KB per
// 128 rows against 4 KB of packed codes, and writing it to shared memory and
// reading it back for the MMA made shared-memory bandwidth the limit.
//
// Operand order: with PERM the dequant writes each group of 8 inputs in the
// order [0,4,1,5,2,6,3,7] (what the magic-number extraction yields without
// byte permutes), and the activation operand was written in the same order
// by its producer (gather_f16 / the SwiGLU epilogue with y_f16); without
// PERM the dequant regroups to natural order with byte permutes.  A dot
// product does not depend on the order of its terms' positions, only on both
// operands using the same one; the tensor core's f32 accumulation order over
// K is not specified either way.
// Tiles are (token block, row block) pairs, enumerated token-block-major so
// blocks working at the same time share the activation tile through L2.
// Every wait is bounded (about one second of SM clock); an expired wait
// records an error code (tf_device_error) and makes every role stop.
// No cluster multicast is used anywhere.
#include <cuda.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "internal.h"
#include "tc_ptx.cuh"

namespace tf {

__device__ int g_tc_error = 0;  // first error code recorded by a bounded wait
// Cycles a pipeline wait may take before the kernel gives up (about one
// second of SM clock; tf_set_wait_limit shortens it for failure tests).
__device__ long long g_wait_cycles = 2000000000LL;

namespace tc {

// Warp roles of a block with G dequant groups of 4 warps (one warp per TMEM
// lane quarter; groups take alternate stages, so while one group waits on a
// barrier or a shared load the others dequantize).  BPS blocks share an SM:
// decode expert tiles run two blocks per SM with 256 TMEM columns each, so two
// MMA issuers run side by side (a small-N MMA is issue-bound, about 50 cycles
// per instruction); dense decode projections and prefill run one block per
// SM owning all 512 columns.
template <int G, int BPS>
struct Roles {
  static constexpr int kDeqGroups = G;
  static constexpr int kDeqWarps = 4 * G;
  static constexpr int kEpiWarps = 4;
  static constexpr int kLoadWarp = kDeqWarps + kEpiWarps;  // packed codes + scales
  static constexpr int kMmaWarp = kLoadWarp + 1;
  static constexpr int kActWarp = kMmaWarp + 1;            // activation tiles
  static constexpr int kThreads = (kActWarp + 1) * 32;
  static constexpr int kBlocksPerSM = BPS;
  static constexpr uint32_t kTmemCols = BPS == 2 ? 256 : 512;
};
constexpr int kM = 128;
constexpr int kKStep = 64;
constexpr int kSK = 8;          // k-steps per scale slot (16 bytes of f16 per row) = one work chunk
constexpr int kMaxSegs = 128;   // per-block segment table
constexpr int kMaxExperts = 256;
constexpr int kFixupParts = 2;
constexpr int kSS = 3;  // scale slots: the loader fetches a chunk's scales one chunk ahead of its codes  // partial tiles read per round trip in the split fixup
constexpr int kACols = kKStep / 2;   // TMEM columns of one k-step of A (two f16 per column)
// Fixed limit of the waits that drain a block's own copies and MMAs before
// it exits (not shortened by tf_set_wait_limit: copies in flight always land).
constexpr long long kDrainCycles = 2000000000LL;

// A block's work item: chunks [kc0, kc1) (a chunk is kSK k-steps) of one
// tile (expert e, token slots s0 .. s0 + cnt, row block rb).  Segments with
// slot < 0 cover every chunk of the tile; the others are parts of a tile
// split across consecutive blocks (split schedule) and meet in the fixup.
struct Seg {
  int e, s0, cnt, rb;
  int kc0, kc1, tile;
  int slot;  // -1: whole tile; else this block's partial slot (2 block + 0 first tile / 1 last tile)
};

struct Params {
  CUtensorMap tm_q0, tm_q1;  // packed codes, box {8*KS words, 128 (or 64) rows}
  CUtensorMap tm_s0, tm_s1;  // scales, box {8 groups, 128 (or 64) rows}
  CUtensorMap tm_b0, tm_b1;  // biases
  CUtensorMap tm_x;          // f16 activations [rows][in], box {64, NT}, 128B swizzle
  const int32_t* offsets;
  const int32_t* active;
  const int32_t* active_count;
  int grouped;
  int experts;  // grouped: experts of the stacked weight (offsets has experts + 1 entries)
  int row_blocks;
  int out;  // rows per expert (per matrix)
  int in;
  int64_t n;  // slots (= activation rows)
  void* y;
  int64_t y_stride;
  const int32_t* y_index;  // EPI_PLAIN output row of each slot (NULL: the slot)
  int y_f16;
  const void* residual;
  int64_t residual_stride;
  // Outputs (and residual) allow 16-byte vector access: the epilogue stages
  // each warp's 32 rows x 16 tokens in shared memory and stores vectors.
  int vec_out;
  // Split schedule (stream-K over chunks): each block takes an equal run of
  // the (tile, chunk) sequence; a tile split across blocks is finished by
  // the last of them to arrive (counters[tile], zero at launch and left zero)
  // from fp32 partials in `partials` (two slots of 128 x NT per block).
  int split;
  float* partials;
  int* counters;
};

// Shared-memory wait control of a block: the abort flag every role polls,
// and the limit and suspend hint of its bounded waits (a test limit below
// the default polls without suspending, so it can expire).
struct WaitCtl {
  volatile int abort;
  uint32_t suspend_ns;
  long long limit;
};
// Bounded wait; false when the phase did not complete in time or another
// role already gave up (abort set).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, WaitCtl* w, int code) {
  const uint32_t susp = w->suspend_ns;
  if (mbar_try(bar, parity, susp)) return true;
  const long long t0 = clock64();
  const long long limit = w->limit;
  while (!mbar_try(bar, parity, susp)) {
    if (w->abort) return false;
    if (clock64() - t0 > limit) {
      atomicCAS(&g_tc_error, 0, code);
      w->abort = 1;
      return false;
    }
  }
  return true;
}
// Wait for a phase that is known to complete (a block's own TMA copy or
// MMA commit) before the block exits, ignoring the abort flag; fixed limit.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return;
  const long long t0 = clock64();
  while (!mbar_try(bar, parity))
    if (clock64() - t0 > kDrainCycles) {
      atomicCAS(&g_tc_error, 0, 51);
      return;
    }
}
// Warp-uniform bounded wait (every lane waits; all agree on the result).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, WaitCtl* w, int code) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, w, code));
}
// Eight codes of one packed word (code i at bits 4i) -> eight f16 weights
// fp16(code*s + b).  The f16 halves of
//   t0 = w & 0x000F000F | 0x6400 (1024 + c0, 1024 + c4)
//   t1 = w & 0x00F000F0 | 0x5400 (  64 + c1,   64 + c5)   [ulp of 64 is 1/16]
//   t2, t3 = the same on w >> 8  (c2, c6) and (c3, c7)
// are exact; subtracting the magic is exact and one HFMA2 rounds c*s + b
// once.  PERM keeps the pairs as they come (order 0,4,1,5,2,6,3,7: one shift
// and four LOP3 per word); otherwise four byte permutes restore 0..7.
template <bool PERM>
__device__ __forceinline__ uint4 dequant8(uint32_t w, __half2 s2, __half2 b2) {
  const uint32_t w8 = w >> 8;
  const uint32_t t0 = (w & 0x000F000Fu) | 0x64006400u;
  const uint32_t t1 = (w & 0x00F000F0u) | 0x54005400u;
  const uint32_t t2 = (w8 & 0x000F000Fu) | 0x64006400u;
  const uint32_t t3 = (w8 & 0x00F000F0u) | 0x54005400u;
  uint32_t q[4];
  __half2 m[4];
  if (PERM) {
    q[0] = t0, q[1] = t1, q[2] = t2, q[3] = t3;
    const __half2 hi = __half2half2(__ushort_as_half(0x6400)), lo = __half2half2(__ushort_as_half(0x5400));
    m[0] = hi, m[1] = lo, m[2] = hi, m[3] = lo;
  } else {
    q[0] = __byte_perm(t0, t1, 0x5410);  // (c0, c1)
    q[1] = __byte_perm(t2, t3, 0x5410);  // (c2, c3)
    q[2] = __byte_perm(t0, t1, 0x7632);  // (c4, c5)
    q[3] = __byte_perm(t2, t3, 0x7632);  // (c6, c7)
    const __half2 mm = __halves2half2(__ushort_as_half(0x6400), __ushort_as_half(0x5400));
    m[0] = m[1] = m[2] = m[3] = mm;
  }
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 n = __hsub2(*reinterpret_cast<const __half2*>(&q[i]), m[i]);
    const __half2 h = __hfma2(n, s2, b2);
    o[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}
// Column of element f in an operand written in the PERM order.
__host__ __device__ __forceinline__ int perm_col(int f) {
  const int q = f & 7;
  return (f & ~7) | ((q & 3) << 1) | (q >> 2);
}

__device__ __forceinline__ uint32_t u4_word(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Block that owns unit u of U units split over `grid` blocks in equal runs
// (block b owns [floor(b U / grid), floor((b + 1) U / grid))).
// 32-bit: the launcher splits only problems with U * grid < 2^31.
__device__ __forceinline__ int unit_owner(int u, int U, int grid) { return ((u + 1) * grid - 1) / U; }
__device__ __forceinline__ int unit_start(int b, int U, int grid) { return b * U / grid; }

template <int NT, int KS, int PK, int SA, int SB, int G, int H, int BPS>
struct Layout {
  static constexpr int kP = kM * 32 * KS;     // packed codes of one stage
  static constexpr int kS = 2 * kM * kSK * 2;  // scales | biases of 8 k-steps
  static constexpr int kB = NT * 128 * KS;     // f16 activation stage
  static constexpr int kOffSeg = 1024;
  static constexpr int kHead = kOffSeg + kMaxSegs * (int)sizeof(Seg);
  static constexpr int kOffS = (kHead + 1023) / 1024 * 1024;
  static constexpr int kOffP = (kOffS + kSS * kS + 1023) / 1024 * 1024;
  static constexpr int kOffB = kOffP + PK * kP;
  static constexpr int kOffE = kOffB + SB * kB;  // epilogue staging: 4 warps x 2 KB
  static constexpr int kBytes = kOffE + 4 * 2048 + 1024;  // + alignment slack
  // TMEM columns: accumulators [0, 2 NT), A stages from 2 NT on.
  static constexpr int kAStage = KS * kACols;
  static constexpr int kACol0 = 2 * NT;
  static_assert(kP % 1024 == 0 && kB % 1024 == 0, "stage sizes keep 1024-byte alignment");
  static_assert(kSK % KS == 0, "a scale slot holds whole stages");
  static_assert(kACol0 + SA * kAStage <= (int)Roles<G * H, BPS>::kTmemCols, "accumulators and A stages fit tensor memory");
  static_assert(4 * (kMaxExperts + 1) * 4 <= PK * kP, "setup expert table fits the code ring");
  static_assert(H == 1 || H == 2, "one or two threads per weight row and k-step");
  // mbarriers (then the TMEM slot and segment count) below the wait control at 448.
  static_assert((2 * PK + 2 * SA + 2 * SB + 2 * kSS + 5) * 8 + 8 <= 448, "barrier block fits below the wait control");
};

// Residual values of the 8 tokens c0 .. c0 + 7 of TMEM lane q's row (0 past
// the segment or the matrix).  The epilogue loads them 8 tokens ahead of
// their use, so the loads overlap the previous tokens' stores; a load always
// precedes the store of the same element, so y may alias residual.
template <typename T>
__device__ __forceinline__ void epi_residual(const Params& p, const Seg& sg, int q, int c0, float* res) {
  const int f = sg.rb * kM + q;
  const int n = f < p.out ? sg.cnt - c0 : 0;  // valid tokens from c0
  const T* r = static_cast<const T*>(p.residual) + ((int64_t)(sg.s0 + c0) * p.residual_stride + f);
#pragma unroll
  for (int i = 0; i < 8; ++i, r += p.residual_stride) res[i] = i < n ? to_f(*r) : 0.f;
}

// y = act(residual + act(acc)) for the 8 tokens c0 .. c0 + 7 of lane q's row.
template <typename T>
__device__ __forceinline__ void epi_residual_store(const Params& p, const Seg& sg, int q, int c0, const float* v,
                                                   const float* res) {
  const int f = sg.rb * kM + q;
  const int n = f < p.out ? sg.cnt - c0 : 0;
  T* y = static_cast<T*>(p.y) + ((int64_t)(sg.s0 + c0) * p.y_stride + f);
#pragma unroll
  for (int i = 0; i < 8; ++i, y += p.y_stride)
    if (i < n) *y = from_f<T>(res[i] + round_act<T>(v[i]));
}

// Epilogue of 16 accumulator columns (tokens c0 .. c0 + 15 of the segment's
// tile) held by TMEM lane q.
template <typename T, int EPI>
__device__ __forceinline__ void epi_apply(const Params& p, const Seg& sg, int q, int c0, const float* v) {
  constexpr bool kSw = EPI == EPI_SWIGLU;
  if (kSw) {
    // Lanes 2j (gate row j) and 2j+1 (up row j) split the 16 tokens: the even
    // lane finishes tokens 0-7, the odd one 8-15, each getting the partner's
    // value with one shuffle.  SiLU uses the fast exponential and division;
    // the result is rounded to the activation dtype like the reference's
    // compiled silu * up.
    const int f = sg.rb * (kM / 2) + (q >> 1);
    const int fo = p.y_f16 ? perm_col(f) : f;  // an f16 operand for the next tensor-core QMM
    const int odd = q & 1;
    bool wide = false;  // a value beyond the f16 range went to the f16 operand
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float mine = odd ? v[8 + i] : v[i];
      const float theirs = __shfl_xor_sync(0xffffffffu, odd ? v[i] : v[8 + i], 1);
      const int tok = c0 + i + 8 * odd;
      if (tok < sg.cnt && f < p.out) {
        const float gg = round_act<T>(odd ? theirs : mine);
        const float uu = round_act<T>(odd ? mine : theirs);
        const float sl = round_act<T>(__fdividef(gg, 1.0f + __expf(-gg)));
        const float hv = round_act<T>(sl * uu);
        const int64_t row = (int64_t)(sg.s0 + tok) * p.y_stride;
        if (p.y_f16) {
          wide |= fabsf(hv) > 65504.f;
          static_cast<__half*>(p.y)[row + fo] = __float2half_rn(hv);
        } else {
          static_cast<T*>(p.y)[row + f] = from_f<T>(hv);
        }
      }
    }
    // The f16 operand of the down projection: a bf16 value beyond the f16
    // range became inf there, which records device error 5.
    if (wide) atomicCAS(&g_tc_error, 0, 5);
  } else if (EPI == EPI_RESIDUAL) {
#pragma unroll
    for (int h = 0; h < 16; h += 8) {
      float res[8];
      epi_residual<T>(p, sg, q, c0 + h, res);
      epi_residual_store<T>(p, sg, q, c0 + h, v + h, res);
    }
  } else {
    const int f = sg.rb * kM + q;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int tok = c0 + i;
      const float vi = v[i];
      if (tok < sg.cnt && f < p.out) {
        const int64_t slot = sg.s0 + tok;
        if (EPI == EPI_F32) {
          static_cast<float*>(p.y)[slot * p.y_stride + f] = round_act<T>(vi);
        } else {
          const int64_t orow = p.y_index ? (int64_t)p.y_index[slot] : slot;
          static_cast<T*>(p.y)[orow * p.y_stride + f] = from_f<T>(vi);
        }
      }
    }
  }
}

// Staged epilogue of 16 accumulator columns (tokens c0 .. c0 + 15) of the
// warp's 32 TMEM lanes: the values go through the warp's 2 KB of shared
// memory so that each lane then stores 16-byte vectors of consecutive
// outputs of one token (the direct form stores one value per token and row;
// at 192-token tiles its per-output instructions starved the epilogue warps
// of issue slots and bounded the whole tile).  Same values as epi_apply.
// res: EPI_RESIDUAL only, the residual vectors of this lane's two (token,
// 8-row) pieces, loaded ahead by the caller (epi_residual_vec).
// Packed fp32 pairs (each lane rounded as the scalar operation).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2eF = 1.4426950408889634f;
// Both values rounded to the activation dtype (one packed conversion).
template <typename T>
__device__ __forceinline__ void round2_act(float& a, float& b);
template <>
__device__ __forceinline__ void round2_act<__half>(float& a, float& b) {
  const float2 f = __half22float2(__floats2half2_rn(a, b));
  a = f.x, b = f.y;
}
template <>
__device__ __forceinline__ void round2_act<__nv_bfloat16>(float& a, float& b) {
  const float2 f = __bfloat1622float2(__floats2bfloat162_rn(a, b));
  a = f.x, b = f.y;
}

template <typename T>
__device__ __forceinline__ void epi_residual_vec(const Params& p, const Seg& sg, int wq, int lane, int c0, uint4* res) {
  const int f0 = sg.rb * kM + wq * 32;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int k = lane + 32 * h, t = k >> 2, g = k & 3;
    res[h] = make_uint4(0, 0, 0, 0);
    if (c0 + t < sg.cnt && f0 + 8 * g < p.out)
      res[h] = ld_v4(static_cast<const T*>(p.residual) + ((int64_t)(sg.s0 + c0 + t) * p.residual_stride + f0 + 8 * g));
  }
}

template <typename T, int EPI>
__device__ __forceinline__ void epi_staged(const Params& p, const Seg& sg, int wq, int lane, int c0, const float* v,
                                           uint8_t* stage, const uint4* res) {
  if (EPI == EPI_SWIGLU) {
    // 16 features (lane pairs) x 16 tokens; the even lane of a pair finishes
    // tokens 0-7, the odd one 8-15 (as epi_apply), two tokens at a time on
    // packed fp32 pairs (the same operations as epi_apply: act-rounded gate
    // and up, SiLU by the fast exponential and reciprocal, act rounding).
    const int base = sg.rb * (kM / 2) + wq * 16;  // the warp's first feature (a multiple of 8)
    const int f = base + (lane >> 1);
    const int col = (p.y_f16 ? perm_col(f) : f) - base;
    const int odd = lane & 1;
    bool wide = false;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i0 = 2 * k;
      const float m0 = odd ? v[8 + i0] : v[i0], m1 = odd ? v[9 + i0] : v[i0 + 1];
      const float x0 = odd ? v[i0] : v[8 + i0], x1 = odd ? v[i0 + 1] : v[9 + i0];
      const float t0 = __shfl_xor_sync(0xffffffffu, x0, 1), t1 = __shfl_xor_sync(0xffffffffu, x1, 1);
      float g0 = odd ? t0 : m0, g1 = odd ? t1 : m1;
      float u0 = odd ? m0 : t0, u1 = odd ? m1 : t1;
      round2_act<T>(g0, g1);
      round2_act<T>(u0, u1);
      const uint64_t gg = f2_pack(g0, g1);
      float e0, e1;
      f2_unpack(f2_mul(gg, f2_pack(-kLog2eF, -kLog2eF)), e0, e1);
      float d0, d1;
      f2_unpack(f2_add(f2_pack(ex2_approx(e0), ex2_approx(e1)), f2_pack(1.f, 1.f)), d0, d1);
      float s0, s1;
      f2_unpack(f2_mul(gg, f2_pack(rcp_approx(d0), rcp_approx(d1))), s0, s1);
      round2_act<T>(s0, s1);
      float h0, h1;
      f2_unpack(f2_mul(f2_pack(s0, s1), f2_pack(u0, u1)), h0, h1);
      round2_act<T>(h0, h1);
      const int t = i0 + 8 * odd;
      if (p.y_f16) {
        if (!std::is_same<T, __half>::value)  // bf16 values beyond the f16 range
          wide |= f < p.out && ((c0 + t < sg.cnt && fabsf(h0) > 65504.f) || (c0 + t + 1 < sg.cnt && fabsf(h1) > 65504.f));
        reinterpret_cast<__half*>(stage)[t * 16 + col] = __float2half_rn(h0);
        reinterpret_cast<__half*>(stage)[(t + 1) * 16 + col] = __float2half_rn(h1);
      } else {
        reinterpret_cast<T*>(stage)[t * 16 + col] = from_f<T>(h0);
        reinterpret_cast<T*>(stage)[(t + 1) * 16 + col] = from_f<T>(h1);
      }
    }
    __syncwarp();
    const int t = lane >> 1, g = lane & 1;
    const uint4 val = *reinterpret_cast<const uint4*>(stage + (t * 16 + 8 * g) * 2);
    if (c0 + t < sg.cnt && base + 8 * g < p.out)
      *reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.y) +
                                ((int64_t)(sg.s0 + c0 + t) * p.y_stride + base + 8 * g) * 2) = val;
    __syncwarp();
    // The f16 operand of the down projection: a bf16 value beyond the f16
    // range became inf there, which records device error 5.
    if (wide) atomicCAS(&g_tc_error, 0, 5);
  } else if (EPI == EPI_F32) {
    float* st = reinterpret_cast<float*>(stage);
#pragma unroll
    for (int i = 0; i < 16; ++i) st[i * 32 + lane] = round_act<T>(v[i]);
    __syncwarp();
    const int f0 = sg.rb * kM + wq * 32;
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const int k = lane + 32 * h, t = k >> 3, g = k & 7;
      const float4 val = *reinterpret_cast<const float4*>(st + t * 32 + 4 * g);
      if (c0 + t < sg.cnt && f0 + 4 * g < p.out)
        *reinterpret_cast<float4*>(static_cast<float*>(p.y) + ((int64_t)(sg.s0 + c0 + t) * p.y_stride + f0 + 4 * g)) =
            val;
    }
    __syncwarp();
  } else {
    T* st = reinterpret_cast<T*>(stage);
#pragma unroll
    for (int i = 0; i < 16; ++i) st[i * 32 + lane] = from_f<T>(v[i]);  // act(acc)
    __syncwarp();
    const int f0 = sg.rb * kM + wq * 32;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int k = lane + 32 * h, t = k >> 2, g = k & 3;
      uint4 val = *reinterpret_cast<const uint4*>(st + t * 32 + 8 * g);
      if (c0 + t < sg.cnt && f0 + 8 * g < p.out) {
        const int64_t slot = sg.s0 + c0 + t;
        if (EPI == EPI_RESIDUAL) {
          float a[8], r[8];
          unpack8<T>(val, a);
          unpack8<T>(res[h], r);
#pragma unroll
          for (int i = 0; i < 8; ++i) a[i] = r[i] + a[i];
          val = pack8<T>(a);
        }
        const int64_t orow = EPI == EPI_PLAIN && p.y_index ? (int64_t)p.y_index[slot] : slot;
        *reinterpret_cast<uint4*>(static_cast<T*>(p.y) + (orow * p.y_stride + f0 + 8 * g)) = val;
      }
    }
    __syncwarp();
  }
}

template <typename T, int EPI, bool PERM, int NT, int KS, int PK, int SA, int SB, int G, int H, int BPS>
__global__ void __launch_bounds__(Roles<G * H, BPS>::kThreads, BPS)
    qmm_tc_kernel(const __grid_constant__ Params p) {
  using L = Layout<NT, KS, PK, SA, SB, G, H, BPS>;
  // G groups of 4 H warps; Roles counts groups of 4 warps.
  using R = Roles<G * H, BPS>;
  constexpr int kDeqWarps = R::kDeqWarps, kEpiWarps = R::kEpiWarps;
  constexpr int kGroupWarps = 4 * H;
  constexpr int kLoadWarp = R::kLoadWarp, kMmaWarp = R::kMmaWarp, kActWarp = R::kActWarp;
  constexpr uint32_t kTmemCols = R::kTmemCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* p_full = reinterpret_cast<uint64_t*>(base);
  uint64_t* p_empty = p_full + PK;
  uint64_t* s_full = p_empty + PK;
  uint64_t* s_empty = s_full + kSS;
  uint64_t* a_full = s_empty + kSS;  // A stage in TMEM written (dequant warps of one group)
  uint64_t* a_empty = a_full + SA;  // A stage read by its MMAs (commit)
  uint64_t* b_full = a_empty + SA;  // activation stage landed (TMA)
  uint64_t* b_empty = b_full + SB;  // activation stage read by its MMAs (commit)
  uint64_t* acc_full = b_empty + SB;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  WaitCtl* wctl = reinterpret_cast<WaitCtl*>(base + 448);
  int* nsegs_s = reinterpret_cast<int*>(tmem_slot + 1);
  int* units_s = reinterpret_cast<int*>(base + 512);
  Seg* segs = reinterpret_cast<Seg*>(base + L::kOffSeg);
  uint8_t* ring_s = base + L::kOffS;  // [kSS slots][s | b][kM rows][8 k-steps] f16
  uint8_t* ring_p = base + L::kOffP;
  uint8_t* ring_b = base + L::kOffB;
  uint8_t* ring_e = base + L::kOffE;
  const int nk = p.in / kKStep;  // a multiple of 8
  const int cpt = nk / kSK;      // chunks per tile
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // ---- setup
  if (tid == 0) {
    for (int i = 0; i < PK; ++i) {
      mbar_init(&p_full[i], 1);
      mbar_init(&p_empty[i], kGroupWarps);
    }
    for (int i = 0; i < kSS; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kDeqWarps);  // every group uses every scale block
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiWarps);
    }
    for (int i = 0; i < SA; ++i) {
      mbar_init(&a_full[i], kGroupWarps);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < SB; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    mbar_init(drain, 1);
    const long long lim = g_wait_cycles;
    wctl->abort = 0;
    wctl->limit = lim;
    wctl->suspend_ns = lim < 2000000000LL ? 0u : kSuspendNs;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (warp == kLoadWarp && lane == 0) {
    // Fetch the tensor maps while the segment table is built.
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_q0)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_s0)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_b0)) : "memory");
    if (EPI == EPI_SWIGLU) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_q1)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_s1)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_b1)) : "memory");
    }
  }
  if (warp == kActWarp && lane == 0)
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_x)) : "memory");
  if (warp == 0) {
    // Segment table.  Grouped problems: every expert's token blocks from one
    // round of independent offset loads (prefix sums in a table that lives
    // in the code ring until the loaders start; experts without routes get
    // no blocks), then every tile found by binary search, one lane per
    // segment.
    int* ex_id = reinterpret_cast<int*>(ring_p);
    int* ex_lo = ex_id + kMaxExperts;
    int* ex_hi = ex_lo + kMaxExperts;
    int* tb_end = ex_hi + kMaxExperts;
    int na = 0;
    int tblocks;
    if (p.grouped) {
      na = p.experts;
      int lo_r[kMaxExperts / 32], hi_r[kMaxExperts / 32];
#pragma unroll
      for (int r = 0; r < kMaxExperts / 32; ++r) {
        const int i = r * 32 + lane;
        lo_r[r] = i < na ? p.offsets[i] : 0;
        hi_r[r] = i < na ? p.offsets[i + 1] : 0;
      }
      int run = 0;
#pragma unroll
      for (int r = 0; r < kMaxExperts / 32; ++r) {
        const int c0 = r * 32;
        if (c0 >= na) break;
        const int i = c0 + lane;
        int nb = 0;
        if (i < na) {
          // Offsets outside [0, n] (a caller's corrupted sort output) are
          // clamped: wrong rows at worst, never an address past the operands.
          const int nrows = (int)p.n;
          const int lo = min(max(lo_r[r], 0), nrows), hi = min(max(hi_r[r], lo), nrows);
          nb = (hi - lo + NT - 1) / NT;
          ex_id[i] = i;
          ex_lo[i] = lo;
          ex_hi[i] = hi;
        }
        int incl = nb;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += v;
        }
        if (i < na) tb_end[i] = run + incl;
        run += __shfl_sync(0xffffffffu, incl, 31);
      }
      tblocks = run;
    } else {
      tblocks = (int)((p.n + NT - 1) / NT);
    }
    __syncwarp();
    const int tiles = tblocks * p.row_blocks;  // < 2^31 (launcher)
    const int grid = (int)gridDim.x;
    int U = 0, u0 = 0, u1 = 0, t_first = 0, t_last = -1;
    int ns;
    if (p.split) {
      U = tiles * cpt;
      u0 = unit_start(blockIdx.x, U, grid);
      u1 = unit_start(blockIdx.x + 1, U, grid);
      if (u1 > u0) {
        t_first = u0 / cpt;
        t_last = (u1 - 1) / cpt;
      }
      ns = t_last - t_first + 1;
    } else {
      ns = (int)blockIdx.x < tiles ? (tiles - 1 - (int)blockIdx.x) / grid + 1 : 0;
    }
    const int nsegs = (int)(ns < kMaxSegs ? ns : kMaxSegs);  // the launcher sizes the grid so ns fits
    for (int j = lane; j < nsegs; j += 32) {
      const int t = p.split ? t_first + j : (int)blockIdx.x + j * grid;
      const int tblock = t / p.row_blocks;
      Seg s;
      s.tile = t;
      s.rb = t - tblock * p.row_blocks;
      if (p.grouped) {
        int lo = 0, hi = na - 1;  // first i with tb_end[i] > tblock
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (tb_end[mid] > tblock)
            hi = mid;
          else
            lo = mid + 1;
        }
        const int first = lo ? tb_end[lo - 1] : 0;
        s.e = ex_id[lo];
        s.s0 = ex_lo[lo] + (tblock - first) * NT;
        s.cnt = min(NT, ex_hi[lo] - s.s0);
      } else {
        s.e = 0;
        s.s0 = tblock * NT;
        s.cnt = (int)((p.n - s.s0) < (int64_t)NT ? (p.n - s.s0) : (int64_t)NT);
      }
      s.kc0 = p.split && t == t_first ? u0 - t * cpt : 0;
      s.kc1 = p.split && t == t_last ? u1 - t * cpt : cpt;
      s.slot = (s.kc0 == 0 && s.kc1 == cpt) ? -1 : 2 * (int)blockIdx.x + (t == t_first ? 0 : 1);
      segs[j] = s;
    }
    __syncwarp();
    if (lane == 0) {
      // A block's split tiles are its first and last; run the last one
      // first too, so that their fixups happen early and the block ends on
      // whole tiles.
      if (nsegs >= 2 && segs[nsegs - 1].slot >= 0) {
        const Seg last = segs[nsegs - 1];
        for (int j = nsegs - 1; j > 0; --j) segs[j] = segs[j - 1];
        segs[0] = last;
      }
      *nsegs_s = nsegs;
      *units_s = U;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const int nsegs = *nsegs_s;
  const uint32_t tmem = *tmem_slot;
  constexpr bool kSw = EPI == EPI_SWIGLU;
  constexpr int kTileRows = kSw ? kM / 2 : kM;  // rows of each weight matrix per tile
  constexpr int kSpb = kSK / KS;                // stages per scale block

  if (warp == kLoadWarp) {
    // ---- code loader: lane 0 streams packed codes (PK stages ahead of the
    // dequant warps) and the scales of every chunk.  Activation tiles have
    // their own warp, so the weight stream never waits on the MMA.
    if (lane == 0) {
      int g = 0;  // stage counter (< 2^31 per block)
      bool ok = true;
      // Scale cursor: the next chunk (segment sj, chunk sc) whose scales to
      // fetch, gsi chunks fetched so far.  Scales run one chunk ahead of the
      // codes, so a group's first stage of a chunk never waits for them
      // behind the previous chunk's code stages.
      int sj = 0, sc = nsegs > 0 ? segs[0].kc0 : 0, gsi = 0;
      auto fetch_scales = [&]() -> bool {
        while (sj < nsegs && sc >= segs[sj].kc1) {
          ++sj;
          if (sj < nsegs) sc = segs[sj].kc0;
        }
        if (sj >= nsegs) return true;
        const Seg& ssg = segs[sj];
        const int row0s = ssg.e * p.out + ssg.rb * kTileRows;
        const int k8 = sc * kSK;
        const int ss = gsi % kSS;
        if (gsi >= kSS && !mbar_wait(&s_empty[ss], (uint32_t)(((gsi / kSS) - 1) & 1), wctl, 11)) return false;
        uint8_t* sdst = ring_s + (size_t)ss * L::kS;
        mbar_expect_tx(&s_full[ss], (uint32_t)L::kS);
        tma_2d(sdst, &p.tm_s0, k8, row0s, &s_full[ss]);
        tma_2d(sdst + kM * kSK * 2, &p.tm_b0, k8, row0s, &s_full[ss]);
        if (kSw) {
          tma_2d(sdst + 64 * kSK * 2, &p.tm_s1, k8, row0s, &s_full[ss]);
          tma_2d(sdst + kM * kSK * 2 + 64 * kSK * 2, &p.tm_b1, k8, row0s, &s_full[ss]);
        }
        ++sc;
        ++gsi;
        return true;
      };
      ok = fetch_scales();
      for (int j = 0; j < nsegs && ok; ++j) {
        const Seg sg = segs[j];
        const int row0 = sg.e * p.out + sg.rb * kTileRows;
        for (int c = sg.kc0; c < sg.kc1 && ok; ++c) {
          const int k8 = c * kSK;
          if (!(ok = fetch_scales())) break;  // the next chunk's
          for (int ks = 0; ks < kSK && ok; ks += KS, ++g) {
            const int ps = g % PK;
            if (g >= PK && !(ok = mbar_wait(&p_empty[ps], (uint32_t)(((g / PK) - 1) & 1), wctl, 12))) break;
            uint8_t* pdst = ring_p + (size_t)ps * L::kP;
            mbar_expect_tx(&p_full[ps], (uint32_t)L::kP);
            tma_2d(pdst, &p.tm_q0, (k8 + ks) * 8, row0, &p_full[ps]);
            if (kSw) tma_2d(pdst + 64 * 32 * KS, &p.tm_q1, (k8 + ks) * 8, row0, &p_full[ps]);
          }
        }
      }
      // Every copy issued into the rings lands before the block may exit
      // (after an expired wait the consumers are gone but the copies are not).
      for (int i = g - 1; i >= 0 && i >= g - PK; --i) mbar_drain(&p_full[i % PK], (uint32_t)((i / PK) & 1));
      for (int i = gsi - 1; i >= 0 && i >= gsi - kSS; --i) mbar_drain(&s_full[i % kSS], (uint32_t)((i / kSS) & 1));
    }
  } else if (warp == kActWarp) {
    // ---- activation loader: lane 0 streams each stage's activation tiles
    // into their own SB-deep ring, independent of the A stages in TMEM.
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int j = 0; j < nsegs && ok; ++j) {
        const Seg sg = segs[j];
        for (int k = sg.kc0 * kSK; k < sg.kc1 * kSK && ok; k += KS, ++g) {
          const int bs = g % SB;
          if (g >= SB && !(ok = mbar_wait(&b_empty[bs], (uint32_t)(((g / SB) - 1) & 1), wctl, 13))) break;
          uint8_t* bdst = ring_b + (size_t)bs * L::kB;
          mbar_expect_tx(&b_full[bs], (uint32_t)L::kB);
#pragma unroll
          for (int kk = 0; kk < KS; ++kk)
            tma_2d(bdst + kk * NT * 128, &p.tm_x, (k + kk) * kKStep, sg.s0, &b_full[bs]);
        }
      }
      for (int i = g - 1; i >= 0 && i >= g - SB; --i) mbar_drain(&b_full[i % SB], (uint32_t)((i / SB) & 1));
    }
  } else if (warp < kDeqWarps) {
    // ---- dequant: group grp (4 H warps) takes stages g = grp, grp + G, ...;
    // in a group warp w owns TMEM lanes (A rows) 32 (w % 4).. and, with
    // H = 2, half kh = w / 4 of every k-step: each thread turns 8 / H packed
    // words per k-step into 32 / H TMEM columns of its row.  Every lane waits
    // on the full barriers (warp-uniform result); one lane per warp arrives
    // on the release barriers after __syncwarp (the barriers count warps).
    static_assert(kSpb % G == 0, "each group takes the same stages of every scale block");
    constexpr int kWords = 8 / H;  // packed words per thread and k-step
    const int grp = warp / kGroupWarps, sub = warp % kGroupWarps;
    const int quarter = sub & 3, kh = sub >> 2;
    const int r = quarter * 32 + lane;
    // A row r <- packed/scale row pr.  SwiGLU tiles interleave gate row j
    // (A row 2j) and up row j (A row 2j+1); the packed and scale slots hold
    // gate rows 0..63 then up rows 64..127.
    const int pr = kSw ? ((r & 1) * 64 + (r >> 1)) : r;
    const uint32_t tlane =
        tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(L::kACol0 + kh * (kACols / H));
    int total = 0;
    for (int j = 0; j < nsegs; ++j) total += (segs[j].kc1 - segs[j].kc0) * kSpb;
    uint4 sv = make_uint4(0, 0, 0, 0), bv = sv;
    bool ok = true;
    for (int g = grp; g < total && ok; g += G) {
      const int sb = g % kSpb;
      const int blk = g / kSpb;
      if (sb == grp % kSpb) {  // this group's first stage of a scale block
        if (!(ok = warp_wait(&s_full[blk % kSS], (uint32_t)((blk / kSS) & 1), wctl, 21))) break;
        const uint8_t* sslot = ring_s + (size_t)(blk % kSS) * L::kS;
        sv = *reinterpret_cast<const uint4*>(sslot + pr * 16);
        bv = *reinterpret_cast<const uint4*>(sslot + kM * kSK * 2 + pr * 16);
      }
      const int ps = g % PK;
      if (!(ok = warp_wait(&p_full[ps], (uint32_t)((g / PK) & 1), wctl, 22))) break;
      uint4 w[KS][kWords / 4];
      const uint8_t* src = ring_p + (size_t)ps * L::kP + pr * (32 * KS) + kh * (32 / H);
#pragma unroll
      for (int kk = 0; kk < KS; ++kk)
#pragma unroll
        for (int i = 0; i < kWords / 4; ++i) w[kk][i] = *reinterpret_cast<const uint4*>(src + kk * 32 + 16 * i);
      const int as = g % SA;
      if (g >= SA && !(ok = warp_wait(&a_empty[as], (uint32_t)(((g / SA) - 1) & 1), wctl, 23))) break;
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        // k-step sb * KS + kk of the scale block: f16 scale and bias.
        const int ki = sb * KS + kk;
        const uint32_t spw = u4_word(sv, ki >> 1), bpw = u4_word(bv, ki >> 1);
        const __half2 sp = *reinterpret_cast<const __half2*>(&spw);
        const __half2 bp = *reinterpret_cast<const __half2*>(&bpw);
        const __half2 s2 = (ki & 1) ? __high2half2(sp) : __low2half2(sp);
        const __half2 b2 = (ki & 1) ? __high2half2(bp) : __low2half2(bp);
#pragma unroll
        for (int h = 0; h < kWords / 4; ++h) {
          const uint32_t wa[4] = {w[kk][h].x, w[kk][h].y, w[kk][h].z, w[kk][h].w};
          uint32_t cols[16];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 d = dequant8<PERM>(wa[i], s2, b2);
            cols[4 * i] = d.x, cols[4 * i + 1] = d.y, cols[4 * i + 2] = d.z, cols[4 * i + 3] = d.w;
          }
          tmem_st16(tlane + (uint32_t)(as * L::kAStage + kk * kACols + h * 16), cols);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      // The packed words and (at the group's last stage of a block) the
      // scales were consumed above, so every lane's shared loads of those
      // slots have completed before they are released (a release right
      // after issuing the loads let the next TMA fill overtake a load still
      // in flight on another lane).
      if (lane == 0) {
        mbar_arrive(&a_full[as]);
        mbar_arrive(&p_empty[ps]);
        if (sb + G >= kSpb) mbar_arrive(&s_empty[blk % kSS]);
      }
    }
  } else if (warp == kMmaWarp) {
    // ---- MMA issuer (whole warp, one elected lane issues)
    const uint32_t leader = elect_one();
    int g = 0;
    bool ok = true;
    for (int j = 0; j < nsegs && ok; ++j) {
      const Seg sg = segs[j];
      const int buf = j & 1;
      if (j >= 2 && !(ok = warp_wait(&acc_empty[buf], (uint32_t)(((j >> 1) - 1) & 1), wctl, 31))) break;
      tc_fence_after();
      const int n_mma = (sg.cnt + 15) / 16 * 16;
      const uint32_t idesc = idesc_f16(kM, n_mma);
      const uint32_t d = tmem + (uint32_t)(buf * NT);
      const int k0 = sg.kc0 * kSK, k1 = sg.kc1 * kSK;
      for (int k = k0; k < k1; k += KS, ++g) {
        const int as = g % SA;
        const int bs = g % SB;
        if (!(ok = warp_wait(&a_full[as], (uint32_t)((g / SA) & 1), wctl, 32))) break;
        if (!(ok = warp_wait(&b_full[bs], (uint32_t)((g / SB) & 1), wctl, 33))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          const uint32_t ta = tmem + (uint32_t)(L::kACol0 + as * L::kAStage + kk * kACols);
          const uint64_t bd = sw128_desc(smem_addr(ring_b + (size_t)bs * L::kB + kk * (NT * 128)));
#pragma unroll
          for (int s = 0; s < kKStep / 16; ++s)  // K=16 slice: 8 TMEM columns of A, +32 B (+2) of B
            mma_f16_ts(leader, d, ta + 8 * s, bd + 2 * s, idesc, (k + kk > k0 || s > 0) ? 1u : 0u);
        }
        mma_commit(leader, &a_empty[as]);
        mma_commit(leader, &b_empty[bs]);
      }
      if (ok) mma_commit(leader, &acc_full[buf]);
    }
    // Every MMA issued by this warp completes before TMEM is released.
    mma_commit(leader, drain);
    mbar_drain(drain, 0);
  } else {
    // ---- epilogue: warps kDeqWarps .. + 3 read TMEM lane quarters 0-3
    const int q = tid - kDeqWarps * 32;  // TMEM lane 0..127
    const int wq = warp & 3;
    const int grid = (int)gridDim.x;
    const int U = *units_s;
    bool ok = true;
    for (int j = 0; j < nsegs && ok; ++j) {
      const Seg sg = segs[j];
      const int buf = j & 1;
      if (!(ok = warp_wait(&acc_full[buf], (uint32_t)((j >> 1) & 1), wctl, 41))) break;
      tc_fence_after();
      const int n_mma = (sg.cnt + 15) / 16 * 16;
      const uint32_t taddr = tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(buf * NT);
      if (sg.slot < 0 && p.vec_out) {
        uint8_t* stage = ring_e + wq * 2048;
        uint4 res[2], nres[2];
        if (EPI == EPI_RESIDUAL) epi_residual_vec<T>(p, sg, wq, lane, 0, nres);
        for (int c0 = 0; c0 < n_mma; c0 += 16) {
          float v[16];
          tmem_ld16(taddr + c0, v);
          if (EPI == EPI_RESIDUAL) {
            res[0] = nres[0], res[1] = nres[1];
            if (c0 + 16 < n_mma) epi_residual_vec<T>(p, sg, wq, lane, c0 + 16, nres);
          }
          epi_staged<T, EPI>(p, sg, wq, lane, c0, v, stage, res);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        continue;
      }
      if (sg.slot < 0) {
        if (EPI == EPI_RESIDUAL) {
          // Residual tiles: each 8 tokens' residual loads issue before the
          // previous 8 tokens' stores.
          float res[8];
          epi_residual<T>(p, sg, q, 0, res);
          for (int c0 = 0; c0 < n_mma; c0 += 16) {
            float v[16];
            tmem_ld16(taddr + c0, v);
#pragma unroll
            for (int h = 0; h < 16; h += 8) {
              float nres[8];
              if (c0 + h + 8 < n_mma) epi_residual<T>(p, sg, q, c0 + h + 8, nres);
              epi_residual_store<T>(p, sg, q, c0 + h, v + h, res);
#pragma unroll
              for (int i = 0; i < 8; ++i) res[i] = nres[i];
            }
          }
        } else {
          for (int c0 = 0; c0 < n_mma; c0 += 16) {
            float v[16];
            tmem_ld16(taddr + c0, v);
            epi_apply<T, EPI>(p, sg, q, c0, v);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
        continue;
      }
      // Part of a split tile: store this block's fp32 partial of the warp's
      // 32 rows, release the accumulator, then count the arrival on this
      // row quarter's counter.  The warp that arrives last for a quarter sums
      // that quarter's parts in k order (block order) from the partials and
      // runs its epilogue; nobody waits for anybody.
      float* mine = p.partials + ((size_t)sg.slot * kM + q) * NT;
#pragma unroll 1
      for (int c0 = 0; c0 < n_mma; c0 += 16) {
        float v[16];
        tmem_ld16(taddr + c0, v);
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          __stcg(reinterpret_cast<float4*>(mine + c0 + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      __threadfence();
      __syncwarp();
      const int b_lo = unit_owner(sg.tile * cpt, U, grid);
      const int b_hi = unit_owner((sg.tile + 1) * cpt - 1, U, grid);
      int parts = 0;  // blocks holding a part (with fewer units than blocks some runs are empty)
      for (int b = b_lo; b <= b_hi; ++b) parts += unit_start(b + 1, U, grid) > unit_start(b, U, grid);
      int* counter = &p.counters[4 * sg.tile + wq];
      int seen = 0;
      if (lane == 0) seen = atomicAdd(counter, 1);
      seen = __shfl_sync(0xffffffffu, seen, 0);
      if (seen != parts - 1) continue;
      __threadfence();
      {
        const int qr = q;
#pragma unroll 1
        for (int c0 = 0; c0 < n_mma; c0 += 16) {
          // Parts in block (= k) order, the loads of up to kFixupParts of
          // them in flight together; an empty run adds +0.
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = 0.f;
#pragma unroll 1
          for (int b0 = b_lo; b0 <= b_hi; b0 += kFixupParts) {
            float4 f[kFixupParts][4];
#pragma unroll
            for (int k = 0; k < kFixupParts; ++k) {
              const int b = b0 + k;
              const int ub = unit_start(b, U, grid);
              const bool has = b <= b_hi && unit_start(b + 1, U, grid) > ub;
              const float* part =
                  p.partials + ((size_t)(2 * b + (has && sg.tile == ub / cpt ? 0 : 1)) * kM + qr) * NT + c0;
#pragma unroll
              for (int i = 0; i < 4; ++i)
                f[k][i] = has ? __ldcg(reinterpret_cast<const float4*>(part + 4 * i)) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int k = 0; k < kFixupParts; ++k)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                v[4 * i] += f[k][i].x;
                v[4 * i + 1] += f[k][i].y;
                v[4 * i + 2] += f[k][i].z;
                v[4 * i + 3] += f[k][i].w;
              }
          }
          if (p.vec_out) {
            uint4 res[2];
            if (EPI == EPI_RESIDUAL) epi_residual_vec<T>(p, sg, wq, lane, c0, res);
            epi_staged<T, EPI>(p, sg, wq, lane, c0, v, ring_e + wq * 2048, res);
          } else {
            epi_apply<T, EPI>(p, sg, qr, c0, v);
          }
        }
      }
      if (lane == 0) *counter = 0;  // left at zero for the next launch
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

}  // namespace tc

namespace {

// cuTensorMapEncodeTiled, fetched from the driver at run time.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D row-major tensor [rows][cols] of `esize`-byte elements, box {bx, by}.
tf_status make_map(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize, int64_t cols, int64_t rows,
                   int64_t row_pitch_bytes, int bx, int by, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return set_error(TF_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (row_pitch_bytes & 15) || ((int64_t)bx * esize) % 16)
    return set_error(TF_ERR_INVALID_ARGUMENT, "qmm_tc: tensor not 16-byte aligned for TMA");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_pitch_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)bx, (cuuint32_t)by};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(TF_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return TF_OK;
}

int num_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

// Weight maps (codes box {8*KS words, rows}, scales/biases box {8, rows}) and
// the launch of one configuration.
template <typename T, int EPI, bool PERM, int NT, int KS, int PK, int SA, int SB, int G, int H, int BPS>
tf_status launch_cfg(tc::Params& p, const QmmProblem& q, int64_t tiles_bound, cudaStream_t s) {
  using L = tc::Layout<NT, KS, PK, SA, SB, G, H, BPS>;
  using R = tc::Roles<G * H, BPS>;
  const bool sw = EPI == EPI_SWIGLU;
  const int in = p.in;
  const int64_t rows_total = (int64_t)(q.w0.experts > 0 ? q.w0.experts : 1) * p.out;
  const int tile_rows = sw ? 64 : 128;
  const tf_affine_weight* ws[2] = {&q.w0, &q.w1};
  CUtensorMap* mq[2] = {&p.tm_q0, &p.tm_q1};
  CUtensorMap* ms[2] = {&p.tm_s0, &p.tm_s1};
  CUtensorMap* mb[2] = {&p.tm_b0, &p.tm_b1};
  for (int i = 0; i < (sw ? 2 : 1); ++i) {
    TF_TRY(make_map(mq[i], ws[i]->q, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, in / 8, rows_total, in / 2, 8 * KS, tile_rows,
                    CU_TENSOR_MAP_SWIZZLE_NONE));
    TF_TRY(make_map(ms[i], ws[i]->scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, in / 64, rows_total, in / 32, tc::kSK,
                    tile_rows, CU_TENSOR_MAP_SWIZZLE_NONE));
    TF_TRY(make_map(mb[i], ws[i]->biases, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, in / 64, rows_total, in / 32, tc::kSK,
                    tile_rows, CU_TENSOR_MAP_SWIZZLE_NONE));
  }
  const void* xs = q.x16 ? q.x16 : q.x;
  const int64_t pitch = q.x16 && q.mode == QMM_GROUPED ? in : q.x_stride;
  TF_TRY(make_map(&p.tm_x, xs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, in, q.n, pitch * 2, 64, NT,
                  CU_TENSOR_MAP_SWIZZLE_128B));
  constexpr size_t smem = L::kBytes;
  static_assert(smem * R::kBlocksPerSM <= 226 * 1024, "qmm_tc: shared memory budget per SM");
  static PerDeviceOnce attr;
  int dev = 0;
  if (attr.needed(&dev)) {
    TF_CUDA(cudaFuncSetAttribute(tc::qmm_tc_kernel<T, EPI, PERM, NT, KS, PK, SA, SB, G, H, BPS>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    TF_CUDA(cudaFuncSetAttribute(tc::qmm_tc_kernel<T, EPI, PERM, NT, KS, PK, SA, SB, G, H, BPS>,
                                 cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    attr.mark(dev);
  }
  const int64_t slots = (int64_t)num_sms() * R::kBlocksPerSM;
  int64_t grid;
  // Split schedule: every block slot takes an equal run of (tile, chunk)
  // units.  It needs a partial slot pair per block, a counter per tile, and
  // a segment table that holds a block's tiles.
  // Only grouped (expert) problems split.  Dense decode projections (fewer
  // tiles than block slots) measured slower split than whole: qkv at B=64
  // 48 vs 23 us per layer.
  p.split = p.grouped && q.partials && q.counters && 4 * tiles_bound <= q.counter_cap &&
            tiles_bound * 16 * slots < 2147483647LL &&
            (size_t)2 * slots * tc::kM * NT * sizeof(float) <= q.partial_bytes &&
            tiles_bound <= (int64_t)(tc::kMaxSegs - 2) * slots;
  if (p.split) {
    grid = slots;
    p.partials = q.partials;
    p.counters = q.counters;
  } else {
    grid = tiles_bound < slots ? tiles_bound : slots;
    const int64_t need = (tiles_bound + tc::kMaxSegs - 1) / tc::kMaxSegs;
    if (grid < need) grid = need;
  }
  if (grid <= 0) return TF_OK;
  if (tiles_bound > 2147483647 / 2) return set_error(TF_ERR_UNSUPPORTED, "qmm_tc: %lld tiles", (long long)tiles_bound);
  tc::qmm_tc_kernel<T, EPI, PERM, NT, KS, PK, SA, SB, G, H, BPS><<<(unsigned)grid, R::kThreads, smem, s>>>(p);
  return check_launch("qmm_tc");
}

template <typename T, int EPI, bool PERM>
tf_status launch_nt(tc::Params& p, const QmmProblem& q, int nt, int64_t tiles_bound, cudaStream_t s) {
  switch (nt) {
    // <NT, KS, PK, SA, SB, G, H, BPS>: expert tiles of a decode batch (many
    // tiles, few tokens) run two blocks per SM (256 TMEM columns each) with
    // two dequant groups of 4 warps; dense projections of a decode batch
    // (few tiles) and prefill tiles one block per SM with two groups of 8
    // warps (two threads per row and k-step), 4 and 2 A stages.
    case 32: return launch_cfg<T, EPI, PERM, 32, 2, 4, 3, 6, 2, 1, 2>(p, q, tiles_bound, s);
    case 64: return launch_cfg<T, EPI, PERM, 64, 2, 4, 4, 4, 2, 2, 1>(p, q, tiles_bound, s);
    default: return launch_cfg<T, EPI, PERM, 192, 2, 4, 2, 3, 2, 2, 1>(p, q, tiles_bound, s);
  }
}

template <typename T, int EPI>
tf_status launch_perm(tc::Params& p, const QmmProblem& q, int nt, int64_t tiles_bound, cudaStream_t s) {
  return q.x16 && q.x16_perm ? launch_nt<T, EPI, true>(p, q, nt, tiles_bound, s)
                             : launch_nt<T, EPI, false>(p, q, nt, tiles_bound, s);
}

}  // namespace

size_t qmm_split_partial_bytes() {
  // The largest configuration that splits: 2 slots x 128 rows x NT fp32 per
  // block, with (NT, blocks per SM) = (32, 2) or (64, 1).
  return (size_t)2 * num_sms() * 2 * tc::kM * 32 * sizeof(float);
}

// Tensor-core QMM.  Activation rows must be contiguous in slot order: for
// dense problems x itself (no x_index), for grouped problems the caller's
// slot-ordered operand (x16 for bf16 models, else x).
tf_status launch_qmm_tc(const QmmProblem& q, cudaStream_t s) {
  if (q.n == 0) return TF_OK;
  if (q.mode == QMM_PER_ROUTE) return set_error(TF_ERR_UNSUPPORTED, "qmm_tc: per-route mode");
  if (q.mode == QMM_DENSE && q.x_index) return set_error(TF_ERR_UNSUPPORTED, "qmm_tc: dense rows must be contiguous");
  if (!q.x16 && (q.act == TF_DTYPE_BF16 || q.mode == QMM_GROUPED))
    return set_error(TF_ERR_STATE, "qmm_tc: needs the f16 operand copy (bf16 or grouped rows)");
  const int in = q.w0.in_features;
  if (in % 512 || in > 8192) return set_error(TF_ERR_UNSUPPORTED, "qmm_tc: in_features %d", in);
  const bool sw = q.epilogue == EPI_SWIGLU;
  const int experts = q.w0.experts > 0 ? q.w0.experts : 1;
  if (q.mode == QMM_GROUPED && experts > tc::kMaxExperts)
    return set_error(TF_ERR_UNSUPPORTED, "qmm_tc: %d experts (at most %d)", experts, tc::kMaxExperts);
  const int out = q.w0.out_features;
  const int tile_rows = sw ? 64 : 128;
  tc::Params p;
  memset(&p, 0, sizeof(p));
  p.offsets = q.offsets;
  p.active = q.active;
  p.active_count = q.active_count;
  p.grouped = q.mode == QMM_GROUPED;
  p.experts = experts;
  p.row_blocks = (out + tile_rows - 1) / tile_rows;
  p.out = out;
  p.in = in;
  p.n = q.n;
  p.y = q.y;
  p.y_stride = q.y_stride;
  p.y_index = q.epilogue == EPI_PLAIN ? q.y_index : nullptr;
  p.y_f16 = q.y_f16;
  p.residual = q.residual;
  p.residual_stride = q.residual_stride;
  {
    const int eb = q.epilogue == EPI_F32 ? 4 : (q.epilogue == EPI_SWIGLU && q.y_f16) ? 2 : act_bytes(q.act);
    const int vw = 16 / eb;  // elements per 16-byte vector
    bool ok = (reinterpret_cast<uintptr_t>(q.y) & 15) == 0 && q.y_stride % vw == 0 && out % vw == 0;
    if (q.epilogue == EPI_RESIDUAL)
      ok = ok && (reinterpret_cast<uintptr_t>(q.residual) & 15) == 0 && q.residual_stride % vw == 0;
    p.vec_out = ok ? 1 : 0;
  }
  // Token tile: about the tokens each weight matrix serves.
  const int64_t per_matrix = p.grouped ? (q.n + experts - 1) / experts : q.n;
  const int nt = per_matrix <= 24 ? 32 : per_matrix <= 64 ? 64 : 192;
  const int64_t token_tiles = p.grouped ? experts + q.n / nt + 1 : (q.n + nt - 1) / nt;
  const int64_t tiles_bound = token_tiles * p.row_blocks;
#define TF_TC_EPI(E)                                                                         \
  return q.act == TF_DTYPE_F16 ? launch_perm<__half, E>(p, q, nt, tiles_bound, s)            \
                               : launch_perm<__nv_bfloat16, E>(p, q, nt, tiles_bound, s);
  switch (q.epilogue) {
    case EPI_PLAIN: TF_TC_EPI(EPI_PLAIN)
    case EPI_SWIGLU: TF_TC_EPI(EPI_SWIGLU)
    case EPI_RESIDUAL: TF_TC_EPI(EPI_RESIDUAL)
    default: TF_TC_EPI(EPI_F32)
  }
#undef TF_TC_EPI
}

// ---------------------------------------------------------------------------
// Operand preparation for the tensor-core path.

// y[i] = f16(x[src(i)]) row by row, src(i) = perm ? perm[i] / div : i, with
// each group of 8 columns in the tensor-core operand order [0,4,1,5,2,6,3,7]
// when `permute` is set.  bf16 -> f16 is exact for |x| in [2^-14, 65504];
// beyond the f16 range the value would become inf, so such rows record error
// code 5.
template <typename Tin>
__global__ void gather_f16_kernel(const Tin* __restrict__ x, int64_t x_stride, const int32_t* __restrict__ perm,
                                  int div, int64_t rows, int width, int permute, __half* __restrict__ y) {
  const int cpr = (width / 8 + blockDim.x - 1) / blockDim.x;  // blocks per row
  const int64_t row = blockIdx.x / cpr;
  const int c = (int)(blockIdx.x % cpr) * blockDim.x + threadIdx.x;
  if (row >= rows || 8 * c >= width) return;
  const int64_t src = perm ? perm[row] / div : row;
  float f[8];
  unpack8<Tin>(ld_v4(x + src * x_stride + 8 * c), f);
  bool bad = false;
#pragma unroll
  for (int j = 0; j < 8; ++j) bad |= fabsf(f[j]) > 65504.f;
  if (bad) atomicCAS(&g_tc_error, 0, 5);
  if (permute) {
    const float g[8] = {f[0], f[4], f[1], f[5], f[2], f[6], f[3], f[7]};
    *reinterpret_cast<uint4*>(y + row * width + 8 * c) = pack8<__half>(g);
  } else {
    *reinterpret_cast<uint4*>(y + row * width + 8 * c) = pack8<__half>(f);
  }
}

tf_status launch_gather_f16(const void* x, int64_t x_stride, int act, const int32_t* perm, int div, int64_t rows,
                            int width, void* y, int permute, cudaStream_t s) {
  if (rows == 0) return TF_OK;
  if (width % 8) return set_error(TF_ERR_SHAPE, "gather_f16: width %d", width);
  const int64_t cpr = (width / 8 + 127) / 128;
  if (rows * cpr > 2147483647) return set_error(TF_ERR_UNSUPPORTED, "gather_f16: too many rows");
  const unsigned grid = (unsigned)(rows * cpr);
  if (act == TF_DTYPE_F16)
    gather_f16_kernel<__half><<<grid, 128, 0, s>>>((const __half*)x, x_stride, perm, div, rows, width, permute,
                                                   (__half*)y);
  else
    gather_f16_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>((const __nv_bfloat16*)x, x_stride, perm, div, rows, width,
                                                          permute, (__half*)y);
  return check_launch("gather_f16");
}

tf_status launch_bf16_to_f16(const void* x, int64_t n, void* y, int permute, cudaStream_t s) {
  if (n == 0) return TF_OK;
  if (n % 2048) return set_error(TF_ERR_SHAPE, "bf16_to_f16: count %lld not a multiple of 2048", (long long)n);
  return launch_gather_f16(x, 2048, TF_DTYPE_BF16, nullptr, 1, n / 2048, 2048, y, permute, s);
}

tf_status make_tma_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize, int64_t cols,
                      int64_t rows, int64_t row_pitch_bytes, int bx, int by, CUtensorMapSwizzle sw) {
  return make_map(m, base, dt, esize, cols, rows, row_pitch_bytes, bx, by, sw);
}

tf_status tc_flags(int** error, long long** wait_cycles) {
  TF_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(error), g_tc_error));
  TF_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(wait_cycles), g_wait_cycles));
  return TF_OK;
}

tf_status set_wait_limit(long long cycles) {
  const long long v = cycles > 0 ? cycles : 2000000000LL;
  TF_CUDA(cudaMemcpyToSymbol(g_wait_cycles, &v, sizeof(v)));
  return TF_OK;
}

int read_tc_error(bool clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int));
  if (clear) {
    const int z = 0;
    cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace tf
