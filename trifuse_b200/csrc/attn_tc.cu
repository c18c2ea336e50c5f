// Prefill attention on the sm_100a tensor cores (tcgen05, TMEM, TMA).
//
// One block per (query block of up to 256 consecutive rows of one request,
// head), split into two halves A (rows 0-127) and B (rows 128-255), each with
// its own softmax warpgroup, so the tensor core computes one half's products
// while the other half's softmax runs: causal softmax(Q K^T * scale) V over
// keys 0 .. pos of the request's own cache, FlashAttention-style in 128-key
// tiles.  Replaces the reference's prefill SDPA (MLXNativeGraniteMoEPrefill.h:
// 446-483, kvcache update_and_attend over the whole chunk with a causal mask).
//
// Roles (320 threads):
//   warps 0-3 / 4-7  softmax of half A / B: thread r owns the half's query
//              row r = TMEM lane r.  They write their f16 Q tile into shared
//              memory, then per key tile read the fp32 scores S from TMEM,
//              mask, take the running max, write P = 2^(S*log2e*scale - m)
//              as f16 into TMEM over S's first 64 columns and add the row
//              sum; at the end they read O from TMEM and write O / l.
//   warp 8     loader: TMA of the K and V tiles (two 64-column boxes each,
//              128-byte swizzle) into a two-stage ring.
//   warp 9     MMA: allocates TMEM; one elected lane issues, per key tile,
//                S_A = Q_A K^T, S_B = Q_B K^T   (Q, K K-major in shared memory)
//                O_A += P_A V, O_B += P_B V      (P in TMEM, V MN-major)
//              a half's next S only after its previous P V has completed
//              (P overlays S).
// TMEM columns: O_A [0,128), O_B [128,256), S_A [256,384), S_B [384,512).
//
// The running max is refreshed lazily: a row keeps the max it used for P
// until a tile raises it by more than 8 (log2 units), so P <= 256 and O is
// rescaled (read, scaled, written back in TMEM) only on such tiles.  The
// result O / l is the same quotient as with the exact max.
//
// Keys past the block's last row hold whatever the cache slot holds (the
// tile reads whole 128-key rows); their scores are masked, and the softmax
// threads of the half whose P V of that tile runs first zero those V rows in
// shared memory before it (a masked P of 0 times a non-finite stale value
// would be NaN).
//
// Every wait is bounded; an expired wait records a code in the tensor-core
// error flag (61-69) and the block winds down without hanging.

#include <cuda.h>

#include "common.cuh"
#include "internal.h"
#include "tc_ptx.cuh"

namespace tf {

tf_status make_tma_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize, int64_t cols,
                      int64_t rows, int64_t row_pitch_bytes, int bx, int by, CUtensorMapSwizzle sw);

namespace {

using namespace tc;

constexpr int kFaRows = 128;   // query rows per half
constexpr int kFaKeys = 128;   // keys per tile
constexpr int kFaD = 128;      // head dim
constexpr int kFaThreads = 320;
constexpr int kFaLoadWarp = 8, kFaMmaWarp = 9;
constexpr int kTileBytes = kFaKeys * kFaD * 2;  // 32 KB: [2 column halves][128 rows][128 B]
constexpr int kHalfBytes = kTileBytes / 2;
constexpr int kOffQ = 0;                           // half X's Q at kOffQ + X * kTileBytes
constexpr int kOffK = 2 * kTileBytes;              // stage s at kOffK + s * 2 * kTileBytes
constexpr int kOffV = 3 * kTileBytes;              // stage s at kOffV + s * 2 * kTileBytes
constexpr int kOffBar = 6 * kTileBytes;            // 192 KB
constexpr int kFaSmem = kOffBar + 256 + 1024;      // + barrier block + alignment slack
constexpr uint32_t kColO = 0, kColS = 256;         // half X: O at kColO + 128 X, S (and P) at kColS + 128 X
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.f;

struct FaParams {
  CUtensorMap tm_k, tm_v;  // f16 [requests * heads * capacity][128], box {64, 128}, 128B swizzle
  const void* q;           // act [rows][heads * 128], roped
  const int4* blocks;      // {first row, rows <= 256, request, first position}
  void* out;               // act [rows][heads * 128]
  int heads, cap;
  float scale_log2;        // scale * log2(e)
  int* err;
  const long long* wait_cycles;
};

struct FaCtl {
  volatile int abort;
  uint32_t suspend_ns;
  long long limit;
};

__device__ __forceinline__ bool fa_wait(uint64_t* bar, uint32_t parity, FaCtl* c, int* err, int code) {
  const uint32_t susp = c->suspend_ns;
  if (mbar_try(bar, parity, susp)) return true;
  const long long t0 = clock64();
  const long long limit = c->limit;
  while (!mbar_try(bar, parity, susp)) {
    if (c->abort) return false;
    if (clock64() - t0 > limit) {
      atomicCAS(err, 0, code);
      c->abort = 1;
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ bool fa_warp_wait(uint64_t* bar, uint32_t parity, FaCtl* c, int* err, int code) {
  return __all_sync(0xffffffffu, fa_wait(bar, parity, c, err, code));
}
// A block's own copies and MMAs always complete: fixed limit, abort ignored.
__device__ __forceinline__ void fa_drain(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try(bar, parity)) return;
  const long long t0 = clock64();
  while (!mbar_try(bar, parity))
    if (clock64() - t0 > 2000000000LL) {
      atomicCAS(err, 0, 69);
      return;
    }
}

// 32 consecutive TMEM columns of this warp's 32 lanes (wait included).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 64 consecutive TMEM columns of this warp's 32 lanes (wait included).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
      "%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// 2^x for x <= 8 on the FMA pipe (x below -127 gives 0): Cody-Waite split
// x = n + f, n = floor(x) (an add with round-down against 1.5 * 2^23 leaves n
// in the low mantissa bits), 2^f on [0, 1) by a cubic fitted here by
// weighted least squares for relative error (max 8.6e-5, below the f16
// rounding of P), and 2^n added to the exponent field.  Takes a quarter of
// the exponentials off the special-function unit.
__device__ __forceinline__ float poly_exp2(float x) {
  x = fmaxf(x, -127.f);
  const float t = __fadd_rd(x, 12582912.f);
  const float n = __fsub_rn(t, 12582912.f);
  const float f = __fsub_rn(x, n);
  float p = fmaf(f, 0.07706641f, 0.22764570f);
  p = fmaf(f, p, 0.69511662f);
  p = fmaf(f, p, 1.f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <typename T>
__global__ void __launch_bounds__(kFaThreads, 1) attn_prefill_tc_kernel(const __grid_constant__ FaParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kOffBar);
  uint64_t* q_full = bars;          // [2] a half's 128 softmax threads wrote its Q
  uint64_t* k_full = bars + 2;      // [2 stages] TMA
  uint64_t* v_full = bars + 4;      // [2 stages] TMA
  uint64_t* kv_empty = bars + 6;    // [2 stages] MMA commit after the tile's P V products
  uint64_t* s_full = bars + 8;      // [2 halves] MMA commit after Q K^T
  uint64_t* p_full = bars + 10;     // [2 halves] 128 softmax threads wrote P (and rescaled O)
  uint64_t* o_done = bars + 12;     // [2 halves] MMA commit after each P V
  uint64_t* drain = bars + 14;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);
  FaCtl* ctl = reinterpret_cast<FaCtl*>(base + kOffBar + 192);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int4 blk = p.blocks[blockIdx.x];
  const int row0 = blk.x, nrows = blk.y, rq = blk.z, pos0 = blk.w;
  const int h = blockIdx.y;
  const int W = p.heads * kFaD;
  const int kend = pos0 + nrows;  // keys [0, kend) exist
  const int ntiles = (kend + kFaKeys - 1) / kFaKeys;
  // Half X: rows [128 X, 128 X + n_x), key tiles [0, nt_x).
  const int n_a = nrows < kFaRows ? nrows : kFaRows, n_b = nrows - n_a;
  const int nt_a = (pos0 + n_a + kFaKeys - 1) / kFaKeys, nt_b = n_b > 0 ? ntiles : 0;
  // The half whose P V of the last tile runs first zeroes its V rows past kend.
  const int zero_half = nt_a == ntiles ? 0 : 1;
  int* err = p.err;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 128);
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(drain, 1);
    const long long lim = *p.wait_cycles;
    ctl->abort = 0;
    ctl->limit = lim;
    ctl->suspend_ns = lim < 2000000000LL ? 0u : kSuspendNs;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kFaMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (warp == kFaLoadWarp && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_k)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&p.tm_v)) : "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int64_t key_row0 = ((int64_t)rq * p.heads + h) * p.cap;  // cache row of key 0

  if (warp == kFaLoadWarp) {
    if (lane == 0) {
      int j = 0;
      bool ok = true;
      for (; j < ntiles && ok; ++j) {
        const int st = j & 1;
        if (j >= 2 && !(ok = fa_wait(&kv_empty[st], (uint32_t)(((j >> 1) - 1) & 1), ctl, err, 61))) break;
        const int y = (int)(key_row0 + (int64_t)j * kFaKeys);
        uint8_t* kd = base + kOffK + st * 2 * kTileBytes;
        uint8_t* vd = base + kOffV + st * 2 * kTileBytes;
        mbar_expect_tx(&k_full[st], (uint32_t)kTileBytes);
        tma_2d(kd, &p.tm_k, 0, y, &k_full[st]);
        tma_2d(kd + kHalfBytes, &p.tm_k, 64, y, &k_full[st]);
        mbar_expect_tx(&v_full[st], (uint32_t)kTileBytes);
        tma_2d(vd, &p.tm_v, 0, y, &v_full[st]);
        tma_2d(vd + kHalfBytes, &p.tm_v, 64, y, &v_full[st]);
      }
      // Copies in flight land before the block exits.
      for (int i = j - 1; i >= 0 && i >= j - 2; --i) {
        fa_drain(&k_full[i & 1], (uint32_t)((i >> 1) & 1), err);
        fa_drain(&v_full[i & 1], (uint32_t)((i >> 1) & 1), err);
      }
    }
  } else if (warp == kFaMmaWarp) {
    const uint32_t leader = elect_one();
    const uint32_t id_qk = idesc_f16(kFaRows, kFaKeys);
    const uint32_t id_pv = idesc_f16(kFaRows, kFaD) | (1u << 16);  // B (V) MN-major
    bool ok = fa_warp_wait(&q_full[0], 0, ctl, err, 62) && (nt_b == 0 || fa_warp_wait(&q_full[1], 0, ctl, err, 62));
    for (int j = 0; j < ntiles && ok; ++j) {
      const int st = j & 1;
      if (!(ok = fa_warp_wait(&k_full[st], (uint32_t)((j >> 1) & 1), ctl, err, 63))) break;
      const uint32_t ka = smem_addr(base + kOffK + st * 2 * kTileBytes);
      for (int x = 0; x < 2 && ok; ++x) {
        if (j >= (x == 0 ? nt_a : nt_b)) continue;
        // P of the half's previous tile overlays S: its P V has completed.
        if (j >= 1 && !(ok = fa_warp_wait(&o_done[x], (uint32_t)((j - 1) & 1), ctl, err, 64))) break;
        tc_fence_after();
        const uint32_t qa = smem_addr(base + kOffQ + x * kTileBytes);
        const uint32_t d = tmem + kColS + (uint32_t)(x * 128);
#pragma unroll
        for (int s = 0; s < kFaD / 16; ++s) {
          const uint32_t off = (uint32_t)((s >> 2) * kHalfBytes + (s & 3) * 32);
          mma_f16(leader, d, sw128_desc(qa + off), sw128_desc(ka + off), id_qk, s > 0 ? 1u : 0u);
        }
        mma_commit(leader, &s_full[x]);
      }
      if (!ok) break;
      if (!(ok = fa_warp_wait(&v_full[st], (uint32_t)((j >> 1) & 1), ctl, err, 65))) break;
      const uint32_t va = smem_addr(base + kOffV + st * 2 * kTileBytes);
      for (int x = 0; x < 2 && ok; ++x) {
        if (j >= (x == 0 ? nt_a : nt_b)) continue;
        if (!(ok = fa_warp_wait(&p_full[x], (uint32_t)(j & 1), ctl, err, 66))) break;
        tc_fence_after();
        const uint32_t pa = tmem + kColS + (uint32_t)(x * 128);
#pragma unroll
        for (int s = 0; s < kFaKeys / 16; ++s)
          mma_f16_ts(leader, tmem + kColO + (uint32_t)(x * 128), pa + 8 * s,
                     sw128_mn_desc(va + s * 2048, kHalfBytes, 1024), id_pv, (j > 0 || s > 0) ? 1u : 0u);
        mma_commit(leader, &o_done[x]);
      }
      if (ok) mma_commit(leader, &kv_empty[st]);
    }
    // Every MMA issued by this warp completes before TMEM is released.
    mma_commit(leader, drain);
    fa_drain(drain, 0, err);
  } else {
    // ---- softmax warps: half x = warp / 4, thread r = the half's query row r = TMEM lane r.
    const int x = warp >> 2;
    const int r = tid - x * 128;
    const int n_x = x == 0 ? n_a : n_b, nt_x = x == 0 ? nt_a : nt_b;
    const int pos_x = pos0 + x * kFaRows;  // position of the half's row 0
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t col_o = kColO + (uint32_t)(x * 128), col_s = kColS + (uint32_t)(x * 128);
    // Q tile -> f16, K-major 128-byte swizzle: row r at r * 128 of each
    // 64-column half, 16-byte chunk c at (c ^ (r & 7)) * 16.
    {
      const T* qrow = static_cast<const T*>(p.q) + (int64_t)(row0 + x * kFaRows + r) * W + h * kFaD;
      uint8_t* qs = base + kOffQ + x * kTileBytes;
#pragma unroll 4
      for (int c = 0; c < 16; ++c) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < n_x) {
          float f[8];
          unpack8<T>(ld_v4(qrow + 8 * c), f);
          v = pack8<__half>(f);
        }
        const int cc = c & 7;
        *reinterpret_cast<uint4*>(qs + (c >> 3) * kHalfBytes + r * 128 + ((cc ^ (r & 7)) << 4)) = v;
      }
      fence_proxy_async();
      mbar_arrive(&q_full[x]);
    }
    // Rows past the half attend as the block's last row (their output is dropped).
    const int pr = pos_x + (r < n_x ? r : (n_x > 0 ? n_x - 1 : 0));
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    int j = 0;
    for (; j < nt_x && ok; ++j) {
      const int st = j & 1;
      if (!(ok = fa_warp_wait(&s_full[x], (uint32_t)(j & 1), ctl, err, 67))) break;
      tc_fence_after();
      float sc[128];
      tmem_ld64(lane_base + col_s, sc);
      tmem_ld64(lane_base + col_s + 64, sc + 64);
      const int lim = pr - j * kFaKeys;  // keys c > lim of this tile are masked
      // Eight independent partial maxima and sums keep the chains short.
      // The max is taken on the raw scores (the scale is positive) and the
      // scale is folded into the exponent's FMA; only tiles that reach past
      // the half's first row need the causal mask.
      float mp[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mp[i] = -INFINITY;
      if ((j + 1) * kFaKeys > pos_x + 1) {
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const float t = c > lim ? -INFINITY : sc[c];
          sc[c] = t;
          mp[c & 7] = fmaxf(mp[c & 7], t);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 128; ++c) mp[c & 7] = fmaxf(mp[c & 7], sc[c]);
      }
      const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7]))) * p.scale_log2;
      float factor = 1.f;  // O and l scale when the max moves
      if (j == 0) {
        m_used = mx;  // finite: key 0 is attended by every row
      } else if (mx > m_used + kRescale) {
        factor = fast_exp2(m_used - mx);
        m_used = mx;
        l *= factor;
      }
      if (j >= 1) {
        // The previous tile's P V is done: O is stable and P may overlay S.
        if (!(ok = fa_warp_wait(&o_done[x], (uint32_t)((j - 1) & 1), ctl, err, 68))) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, factor != 1.f)) {
#pragma unroll 1
          for (int c = 0; c < 128; c += 32) {
            float o[32];
            tmem_ld32(lane_base + col_o + c, o);
            uint32_t w[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(o[i] * factor);
            tmem_st16(lane_base + col_o + c, w);
            tmem_st16(lane_base + col_o + c + 16, w + 16);
          }
        }
      }
      // P in two halves of 64 keys (32 TMEM columns each) over S's first 64
      // columns; one exponential in four on the FMA pipe (the special-function
      // unit takes eight cycles per warp instruction; the cubic nine issue
      // slots).
      // The exponent arguments and the row sums run on packed fp32 pairs
      // (fma.rn / add.rn .f32x2, each lane rounded as the scalar op).
      const uint64_t sl2 = f2_pack(p.scale_log2, p.scale_log2), nm = f2_pack(-m_used, -m_used);
      uint64_t sp[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) sp[i] = 0ull;  // (+0, +0)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int k0 = 64 * half + 2 * c;
          float x0, x1;
          f2_unpack(f2_fma(f2_pack(sc[k0], sc[k0 + 1]), sl2, nm), x0, x1);
          const float a = fast_exp2(x0), b = (c & 1) ? poly_exp2(x1) : fast_exp2(x1);
          sp[c & 3] = f2_add(sp[c & 3], f2_pack(a, b));
          pk[c] = pack_half2(a, b);
        }
        tmem_st16(lane_base + col_s + 32 * half, pk);
        tmem_st16(lane_base + col_s + 32 * half + 16, pk + 16);
      }
      float s8[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) f2_unpack(sp[i], s8[2 * i], s8[2 * i + 1]);
      l += ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7]));
      tmem_st_wait();
      if (x == zero_half && j == ntiles - 1 && (j + 1) * kFaKeys > kend) {
        // Last tile: zero the V rows of keys that do not exist yet.
        if (!(ok = fa_warp_wait(&v_full[st], (uint32_t)((j >> 1) & 1), ctl, err, 69))) break;
        if (j * kFaKeys + r >= kend) {
          uint8_t* vrow = base + kOffV + st * 2 * kTileBytes + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            *reinterpret_cast<uint4*>(vrow + 16 * c) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(vrow + kHalfBytes + 16 * c) = make_uint4(0, 0, 0, 0);
          }
        }
        fence_proxy_async();
      }
      tc_fence_before();
      mbar_arrive(&p_full[x]);
    }
    if (ok && nt_x > 0 && fa_warp_wait(&o_done[x], (uint32_t)((nt_x - 1) & 1), ctl, err, 68)) {
      tc_fence_after();
      const float inv = 1.f / l;
      T* orow = static_cast<T*>(p.out) + (int64_t)(row0 + x * kFaRows + r) * W + h * kFaD;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        float o[32];
        tmem_ld32(lane_base + col_o + c, o);
        if (r < n_x) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float f[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) f[k] = o[i + k] * inv;
            *reinterpret_cast<uint4*>(orow + c + i) = pack8<T>(f);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kFaMmaWarp)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

}  // namespace

size_t attn_prefill_tc_smem() { return kFaSmem; }

// Prefill attention over query blocks of <= 256 rows (AttnProblem::qblocks)
// with the roped queries q (act [rows][heads * 128]).
tf_status launch_attn_prefill_tc(const AttnProblem& a, const void* q, cudaStream_t s) {
  if (a.nqblocks <= 0) return TF_OK;
  const int64_t cache_rows = (int64_t)a.cache_requests * a.heads * a.capacity;
  if (cache_rows > 2147483647LL - kFaKeys)
    return set_error(TF_ERR_UNSUPPORTED, "attention: cache of %lld rows", (long long)cache_rows);
  FaParams p;
  memset(&p, 0, sizeof(p));
  TF_TRY(make_tma_2d(&p.tm_k, a.k_cache, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kFaD, cache_rows, kFaD * 2, 64, kFaKeys,
                     CU_TENSOR_MAP_SWIZZLE_128B));
  TF_TRY(make_tma_2d(&p.tm_v, a.v_cache, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kFaD, cache_rows, kFaD * 2, 64, kFaKeys,
                     CU_TENSOR_MAP_SWIZZLE_128B));
  p.q = q;
  p.blocks = a.qblocks;
  p.out = a.out;
  p.heads = a.heads;
  p.cap = a.capacity;
  p.scale_log2 = a.scale * kLog2e;
  TF_TRY(tc_flags(&p.err, const_cast<long long**>(&p.wait_cycles)));
  dim3 grid((unsigned)a.nqblocks, (unsigned)a.heads);
  if (a.act == TF_DTYPE_F16) {
    static PerDeviceOnce attr;
    int dev = 0;
    if (attr.needed(&dev)) {
      TF_CUDA(cudaFuncSetAttribute(attn_prefill_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kFaSmem));
      attr.mark(dev);
    }
    attn_prefill_tc_kernel<__half><<<grid, kFaThreads, kFaSmem, s>>>(p);
  } else {
    static PerDeviceOnce attr;
    int dev = 0;
    if (attr.needed(&dev)) {
      TF_CUDA(cudaFuncSetAttribute(attn_prefill_tc_kernel<__nv_bfloat16>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kFaSmem));
      attr.mark(dev);
    }
    attn_prefill_tc_kernel<__nv_bfloat16><<<grid, kFaThreads, kFaSmem, s>>>(p);
  }
  return check_launch("attn_prefill_tc");
}

}  // namespace tf
