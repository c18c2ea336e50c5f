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
// Persistent, warp-specialized block (448 threads, one block per SM):
//   warp 12 (loader)  one thread issues every TMA: packed codes of a k-step
//                     (box 8 words x 128 rows) into a PK-deep ring, the
//                     tile's scales/biases (two slots), and the activation
//                     tile (box 64 x NT, 128B-swizzled = the MMA's K-major
//                     layout) into an SB-deep ring.
//   warps 0-7 (dequant) two threads per A row turn 16 packed bytes into 32
//                     f16 weights (magic-number half2 extraction + HFMA2)
//                     and store them 128B-swizzled into an SA-deep A ring.
//   warp 13 (MMA)     allocates 2 x NT TMEM columns; lane 0 issues
//                     tcgen05.mma (4 x K=16 per k-step) into one of two
//                     accumulators and commits stage releases.
//   warps 8-11 (epilogue) tcgen05.ld the finished accumulator while the next
//                     tile accumulates into the other one; SwiGLU tiles keep
//                     gate row j and up row j in adjacent TMEM lanes, so one
//                     shuffle pairs them.
// Tiles are (token block, row block) pairs, enumerated token-block-major so
// blocks working at the same time share the activation tile through L2.
// Every wait is bounded (about one second of SM clock); an expired wait
// records an error code (tf_device_error) and makes every role stop.
// No cluster multicast is used anywhere.
#include <cuda.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace tf {

__device__ int g_tc_error = 0;  // first error code recorded by a bounded wait

namespace tc {

constexpr int kDeqWarps = 8;
constexpr int kEpiWarps = 4;
constexpr int kLoadWarp = kDeqWarps + kEpiWarps;  // 12
constexpr int kMmaWarp = kLoadWarp + 1;           // 13
constexpr int kThreads = (kMmaWarp + 1) * 32;     // 448
constexpr int kDeqThreads = kDeqWarps * 32;
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kM = 128;
constexpr int kKStep = 64;
constexpr int kMaxTiles = 256;  // per-block tile table
constexpr long long kWaitCycles = 2000000000LL;

struct TileInfo {
  int e, s0, cnt, rb;
};

struct Params {
  CUtensorMap tm_q0, tm_q1;  // packed codes, box {8 words, 128 (or 64) rows}
  CUtensorMap tm_s0, tm_s1;  // scales, box {groups, 128 (or 64) rows}
  CUtensorMap tm_b0, tm_b1;  // biases
  CUtensorMap tm_x;          // f16 activations [rows][in], box {64, NT}, 128B swizzle
  const int32_t* offsets;
  const int32_t* active;
  const int32_t* active_count;
  int grouped;
  int row_blocks;
  int out;  // rows per expert (per matrix)
  int in;
  int64_t n;  // slots (= activation rows)
  int64_t tiles_bound;
  void* y;
  int64_t y_stride;
  int y_f16;
  const void* residual;
  int64_t residual_stride;
};

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; false when the phase did not complete in time or another
// role already gave up (*abort set).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (*abort) return false;
    if (clock64() - t0 > kWaitCycles) {
      atomicCAS(&g_tc_error, 0, code);
      *abort = 1;
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major, 128-byte swizzled operand descriptor (rows of 128 B, 8-row groups
// 1024 B apart; start address advanced by 32 B per K=16 slice).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
  d |= (uint64_t)1 << 16;                   // leading byte offset (unused for SW128 K-major)
  d |= (uint64_t)(1024u >> 4) << 32;        // stride byte offset
  d |= (uint64_t)1 << 46;                   // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                   // SWIZZLE_128B
  return d;
}
// kind::f16 instruction descriptor: f16 x f16 -> f32, K-major A and B.
__device__ __forceinline__ uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  uint32_t m0 = 0, m1 = 0, m2 = 0, m3 = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(m0), "r"(m1), "r"(m2), "r"(m3)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Eight codes of one packed word -> eight f16 weights fp16(code*s + b) in k
// order.  (w >> 4i) & 0x000F000F | 0x64006400 is the f16 pair (1024 + c_i,
// 1024 + c_{i+4}); byte_perm regroups the pairs as (c0,c1) (c2,c3) (c4,c5)
// (c6,c7); subtracting 1024 is exact and one HFMA2 rounds c*s + b once.
__device__ __forceinline__ uint4 dequant8(uint32_t w, __half2 s2, __half2 b2) {
  const uint32_t t0 = (w & 0x000F000Fu) | 0x64006400u;
  const uint32_t t1 = ((w >> 4) & 0x000F000Fu) | 0x64006400u;
  const uint32_t t2 = ((w >> 8) & 0x000F000Fu) | 0x64006400u;
  const uint32_t t3 = ((w >> 12) & 0x000F000Fu) | 0x64006400u;
  const uint32_t q[4] = {__byte_perm(t0, t1, 0x5410), __byte_perm(t2, t3, 0x5410), __byte_perm(t0, t1, 0x7632),
                         __byte_perm(t2, t3, 0x7632)};
  const __half2 k1024 = __half2half2(__ushort_as_half(0x6400));
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 n = __hsub2(*reinterpret_cast<const __half2*>(&q[i]), k1024);
    const __half2 h = __hfma2(n, s2, b2);
    o[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Tile t -> (expert, first slot, token count, row block); e = -1 past the end.
// Must be called by a full warp (grouped lookup scans 32 experts per round).
__device__ TileInfo lookup_tile(const Params& p, int64_t t, int nt, int lane) {
  TileInfo ti{-1, 0, 0, (int)(t % p.row_blocks)};
  const int64_t tblock = t / p.row_blocks;
  if (!p.grouped) {
    const int64_t nblk = (p.n + nt - 1) / nt;
    if (tblock < nblk) {
      ti.e = 0;
      ti.s0 = (int)(tblock * nt);
      ti.cnt = (int)((p.n - ti.s0) < (int64_t)nt ? (p.n - ti.s0) : (int64_t)nt);
    }
    return ti;
  }
  const int na = *p.active_count;
  int64_t base = 0;
  for (int c0 = 0; c0 < na && ti.e < 0; c0 += 32) {
    const int i = c0 + lane;
    int ex = -1, lo = 0, hi = 0;
    if (i < na) {
      ex = p.active[i];
      lo = p.offsets[ex];
      hi = p.offsets[ex + 1];
    }
    const int nb = ex >= 0 ? (hi - lo + nt - 1) / nt : 0;
    int incl = nb;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    const unsigned hit = __ballot_sync(0xffffffffu, ex >= 0 && base + incl > tblock);
    if (hit) {
      const int src = __ffs(hit) - 1;
      const int ex_s = __shfl_sync(0xffffffffu, ex, src);
      const int lo_s = __shfl_sync(0xffffffffu, lo, src);
      const int hi_s = __shfl_sync(0xffffffffu, hi, src);
      const int first = (int)(base + __shfl_sync(0xffffffffu, incl - nb, src));
      ti.e = ex_s;
      ti.s0 = lo_s + (int)(tblock - first) * nt;
      ti.cnt = min(nt, hi_s - ti.s0);
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
  return ti;
}

template <int NT, int PK, int SA, int SB>
struct Layout {
  static constexpr int kP = kM * 32;   // packed codes of one k-step
  static constexpr int kA = kM * 128;  // f16 A tile
  static constexpr int kB = NT * 128;  // f16 activation tile
  static constexpr int kHead = 1024 + kMaxTiles * 16;
  __host__ __device__ static size_t scales(int in) { return (size_t)2 * 2 * kM * (in / 64) * 2; }
  __host__ __device__ static size_t off_scales() { return kHead; }
  __host__ __device__ static size_t off_p(int in) { return (kHead + scales(in) + 1023) / 1024 * 1024; }
  __host__ __device__ static size_t off_a(int in) { return off_p(in) + (size_t)PK * kP; }
  __host__ __device__ static size_t off_b(int in) { return off_a(in) + (size_t)SA * kA; }
  __host__ __device__ static size_t bytes(int in) { return off_b(in) + (size_t)SB * kB + 1024; }
};

template <typename T, int EPI, int NT, int PK, int SA, int SB>
__global__ void __launch_bounds__(kThreads, 1) qmm_tc_kernel(const __grid_constant__ Params p) {
  using L = Layout<NT, PK, SA, SB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* p_full = reinterpret_cast<uint64_t*>(base);
  uint64_t* p_empty = p_full + PK;
  uint64_t* s_full = p_empty + PK;
  uint64_t* s_empty = s_full + 2;
  uint64_t* a_full = s_empty + 2;
  uint64_t* a_empty = a_full + SA;
  uint64_t* b_full = a_empty + SA;
  uint64_t* b_empty = b_full + SB;
  uint64_t* acc_full = b_empty + SB;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* ntiles_s = const_cast<int*>(abort_flag) + 1;
  TileInfo* table = reinterpret_cast<TileInfo*>(base + 1024);
  __half* scl = reinterpret_cast<__half*>(base + L::off_scales());  // [2 slots][s | b][kM][G]
  uint8_t* ring_p = base + L::off_p(p.in);
  uint8_t* ring_a = base + L::off_a(p.in);
  uint8_t* ring_b = base + L::off_b(p.in);
  const int G = p.in / 64;
  const int nk = p.in / kKStep;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr uint32_t kTmemCols = 2 * NT < 32 ? 32 : 2 * NT;

  // ---- setup
  if (tid == 0) {
    for (int i = 0; i < PK; ++i) {
      mbar_init(&p_full[i], 1);
      mbar_init(&p_empty[i], kDeqThreads);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kDeqThreads);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiThreads);
    }
    for (int i = 0; i < SA; ++i) {
      mbar_init(&a_full[i], kDeqThreads);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < SB; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (warp == 0) {
    // This block's tiles: t = blockIdx.x + i * gridDim.x while t < tiles_bound.
    int n = 0;
    for (int64_t t = blockIdx.x; t < p.tiles_bound && n < kMaxTiles; t += gridDim.x) {
      const TileInfo ti = lookup_tile(p, t, NT, lane);
      if (ti.e < 0) break;  // tiles are enumerated in order; later ones are past the end too
      if (lane == 0) table[n] = ti;
      ++n;
    }
    if (lane == 0) *ntiles_s = n;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const int ntiles = *ntiles_s;
  const uint32_t tmem = *tmem_slot;
  constexpr bool kSw = EPI == EPI_SWIGLU;
  constexpr int kTileRows = kSw ? kM / 2 : kM;  // rows of each weight matrix per tile

  if (warp == kLoadWarp) {
    // ---- loader: lane 0 streams packed codes (PK ahead of the dequant warps)
    // and each tile's scales; lane 1 streams activation tiles (SB ahead of
    // the MMA).  Separate issuers keep the weight stream from waiting on the
    // MMA, so up to PK k-steps of codes are in flight.
    if (lane == 0) {
      int64_t g = 0;
      bool ok = true;
      for (int li = 0; li < ntiles && ok; ++li) {
        const TileInfo ti = table[li];
        const int row0 = ti.e * p.out + ti.rb * kTileRows;
        const int ss = li & 1;
        if (li >= 2) ok = mbar_wait(&s_empty[ss], ((li >> 1) - 1) & 1, abort_flag, 11);
        if (!ok) break;
        __half* sdst = scl + (size_t)ss * 2 * kM * G;
        mbar_expect_tx(&s_full[ss], (uint32_t)(2 * kM * G * 2));
        tma_2d(sdst, &p.tm_s0, 0, row0, &s_full[ss]);
        tma_2d(sdst + (size_t)kM * G, &p.tm_b0, 0, row0, &s_full[ss]);
        if (kSw) {
          tma_2d(sdst + (size_t)64 * G, &p.tm_s1, 0, row0, &s_full[ss]);
          tma_2d(sdst + (size_t)kM * G + (size_t)64 * G, &p.tm_b1, 0, row0, &s_full[ss]);
        }
        for (int k = 0; k < nk && ok; ++k, ++g) {
          const int ps = (int)(g % PK);
          if (g >= PK) ok = mbar_wait(&p_empty[ps], (uint32_t)(((g / PK) - 1) & 1), abort_flag, 12);
          if (!ok) break;
          uint8_t* pdst = ring_p + (size_t)ps * L::kP;
          mbar_expect_tx(&p_full[ps], (uint32_t)L::kP);
          tma_2d(pdst, &p.tm_q0, k * 8, row0, &p_full[ps]);
          if (kSw) tma_2d(pdst + 64 * 32, &p.tm_q1, k * 8, row0, &p_full[ps]);
        }
      }
    } else if (lane == 1) {
      int64_t g = 0;
      bool ok = true;
      for (int li = 0; li < ntiles && ok; ++li) {
        const int s0 = table[li].s0;
        for (int k = 0; k < nk && ok; ++k, ++g) {
          const int bs = (int)(g % SB);
          if (g >= SB) ok = mbar_wait(&b_empty[bs], (uint32_t)(((g / SB) - 1) & 1), abort_flag, 13);
          if (!ok) break;
          mbar_expect_tx(&b_full[bs], (uint32_t)L::kB);
          tma_2d(ring_b + (size_t)bs * L::kB, &p.tm_x, k * kKStep, s0, &b_full[bs]);
        }
      }
    }
  } else if (warp < kDeqWarps) {
    // ---- dequant: thread pair per A row, 4 words each per k-step
    const int r = tid >> 1, h = tid & 1;
    // A row r <- packed/scale row pr.  SwiGLU tiles interleave gate row j
    // (A row 2j) and up row j (A row 2j+1); the packed slot holds gate rows
    // 0..63 then up rows 64..127.
    const int pr = kSw ? ((r & 1) * 64 + (r >> 1)) : r;
    int64_t g = 0;
    bool ok = true;
    for (int li = 0; li < ntiles && ok; ++li) {
      const int ss = li & 1;
      ok = mbar_wait(&s_full[ss], (li >> 1) & 1, abort_flag, 21);
      if (!ok) break;
      const __half* srow = scl + (size_t)ss * 2 * kM * G + (size_t)pr * G;
      const __half* brow = srow + (size_t)kM * G;
      for (int k = 0; k < nk; ++k, ++g) {
        const int ps = (int)(g % PK);
        if (!(ok = mbar_wait(&p_full[ps], (uint32_t)((g / PK) & 1), abort_flag, 22))) break;
        const uint4 words = *reinterpret_cast<const uint4*>(ring_p + (size_t)ps * L::kP + pr * 32 + h * 16);
        const __half2 s2 = __half2half2(srow[k]);
        const __half2 b2 = __half2half2(brow[k]);
        mbar_arrive(&p_empty[ps]);
        const int as = (int)(g % SA);
        if (g >= SA && !(ok = mbar_wait(&a_empty[as], (uint32_t)(((g / SA) - 1) & 1), abort_flag, 23))) break;
        uint8_t* arow = ring_a + (size_t)as * L::kA + r * 128;
        const uint32_t wv[4] = {words.x, words.y, words.z, words.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int ch = 4 * h + i;
          *reinterpret_cast<uint4*>(arow + ((ch ^ (r & 7)) << 4)) = dequant8(wv[i], s2, b2);
        }
        fence_proxy_async();
        mbar_arrive(&a_full[as]);
      }
      if (ok) mbar_arrive(&s_empty[ss]);
    }
  } else if (warp == kMmaWarp) {
    // ---- MMA issuer
    if (lane == 0) {
      int64_t g = 0;
      bool ok = true;
      for (int li = 0; li < ntiles && ok; ++li) {
        const TileInfo ti = table[li];
        const int buf = li & 1;
        if (li >= 2 && !(ok = mbar_wait(&acc_empty[buf], ((li >> 1) - 1) & 1, abort_flag, 31))) break;
        tc_fence_after();
        const int n_mma = (ti.cnt + 15) / 16 * 16;
        const uint32_t idesc = idesc_f16(kM, n_mma);
        const uint32_t d = tmem + (uint32_t)(buf * NT);
        for (int k = 0; k < nk; ++k, ++g) {
          const int as = (int)(g % SA), bs = (int)(g % SB);
          if (!(ok = mbar_wait(&a_full[as], (uint32_t)((g / SA) & 1), abort_flag, 32))) break;
          if (!(ok = mbar_wait(&b_full[bs], (uint32_t)((g / SB) & 1), abort_flag, 33))) break;
          tc_fence_after();
          const uint32_t aa = smem_addr(ring_a + (size_t)as * L::kA);
          const uint32_t ba = smem_addr(ring_b + (size_t)bs * L::kB);
#pragma unroll
          for (int j = 0; j < kKStep / 16; ++j)
            mma_f16(d, sw128_desc(aa + 32 * j), sw128_desc(ba + 32 * j), idesc, (k > 0 || j > 0) ? 1u : 0u);
          mma_commit(&a_empty[as]);
          mma_commit(&b_empty[bs]);
        }
        if (ok) mma_commit(&acc_full[buf]);
      }
      // Every MMA issued by this thread completes before TMEM is released.
      mma_commit(drain);
      mbar_wait(drain, 0, abort_flag, 34);
    }
  } else {
    // ---- epilogue: warps 8-11 read TMEM lane quarters 0-3
    const int q = tid - kDeqWarps * 32;  // TMEM lane 0..127
    const int wq = warp & 3;
    bool ok = true;
    for (int li = 0; li < ntiles && ok; ++li) {
      const TileInfo ti = table[li];
      const int buf = li & 1;
      ok = mbar_wait(&acc_full[buf], (li >> 1) & 1, abort_flag, 41);
      // Keep every thread of the warp on the same path for tcgen05.ld.
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const int n_mma = (ti.cnt + 15) / 16 * 16;
      const uint32_t taddr = tmem + ((uint32_t)(wq * 32) << 16) + (uint32_t)(buf * NT);
      for (int c0 = 0; c0 < n_mma; c0 += 16) {
        float v[16];
        tmem_ld16(taddr + c0, v);
        if (kSw) {
          const int f = ti.rb * (kM / 2) + (q >> 1);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float other = __shfl_xor_sync(0xffffffffu, v[i], 1);
            const int tok = c0 + i;
            if ((q & 1) == 0 && tok < ti.cnt && f < p.out) {
              const float gg = round_act<T>(v[i]);
              const float uu = round_act<T>(other);
              const float sl = round_act<T>(gg / (1.0f + expf(-gg)));
              const float hv = round_act<T>(sl * uu);
              const int64_t at = (int64_t)(ti.s0 + tok) * p.y_stride + f;
              if (p.y_f16)
                static_cast<__half*>(p.y)[at] = __float2half_rn(hv);
              else
                static_cast<T*>(p.y)[at] = from_f<T>(hv);
            }
          }
        } else {
          const int f = ti.rb * kM + q;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int tok = c0 + i;
            if (tok < ti.cnt && f < p.out) {
              const int64_t slot = ti.s0 + tok;
              if (EPI == EPI_F32) {
                static_cast<float*>(p.y)[slot * p.y_stride + f] = round_act<T>(v[i]);
              } else if (EPI == EPI_RESIDUAL) {
                const float res = to_f(static_cast<const T*>(p.residual)[slot * p.residual_stride + f]);
                static_cast<T*>(p.y)[slot * p.y_stride + f] = from_f<T>(res + round_act<T>(v[i]));
              } else {
                static_cast<T*>(p.y)[slot * p.y_stride + f] = from_f<T>(v[i]);
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
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

template <typename T, int EPI, int NT, int PK, int SA, int SB>
tf_status launch_cfg(const tc::Params& p, cudaStream_t s) {
  using L = tc::Layout<NT, PK, SA, SB>;
  const size_t smem = L::bytes(p.in);
  if (smem > 227 * 1024) return set_error(TF_ERR_UNSUPPORTED, "qmm_tc: %zu bytes of shared memory", smem);
  static size_t attr = 0;
  if (smem > attr) {
    TF_CUDA(cudaFuncSetAttribute(tc::qmm_tc_kernel<T, EPI, NT, PK, SA, SB>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    attr = smem;
  }
  int64_t grid = p.tiles_bound < num_sms() ? p.tiles_bound : num_sms();
  const int64_t need = (p.tiles_bound + tc::kMaxTiles - 1) / tc::kMaxTiles;
  if (grid < need) grid = need;
  if (grid <= 0) return TF_OK;
  tc::qmm_tc_kernel<T, EPI, NT, PK, SA, SB><<<(unsigned)grid, tc::kThreads, smem, s>>>(p);
  return check_launch("qmm_tc");
}

template <typename T, int EPI>
tf_status launch_nt(tc::Params& p, const QmmProblem& q, int nt, int64_t tiles_bound, cudaStream_t s) {
  const int in = q.w0.in_features;
  const void* xs = q.x16 ? q.x16 : q.x;
  const int64_t pitch = q.x16 && q.mode == QMM_GROUPED ? in : q.x_stride;
  TF_TRY(make_map(&p.tm_x, xs, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, in, q.n, pitch * 2, 64, nt,
                  CU_TENSOR_MAP_SWIZZLE_128B));
  p.tiles_bound = tiles_bound;
  switch (nt) {
    case 32: return launch_cfg<T, EPI, 32, 8, 4, 8>(p, s);
    case 64: return launch_cfg<T, EPI, 64, 8, 4, 6>(p, s);
    default: return launch_cfg<T, EPI, 256, 4, 3, 3>(p, s);
  }
}

}  // namespace

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
  const int out = q.w0.out_features;
  const int64_t rows_total = (int64_t)experts * out;
  const int tile_rows = sw ? 64 : 128;
  tc::Params p;
  memset(&p, 0, sizeof(p));
  TF_TRY(make_map(&p.tm_q0, q.w0.q, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, in / 8, rows_total, in / 2, 8, tile_rows,
                  CU_TENSOR_MAP_SWIZZLE_NONE));
  TF_TRY(make_map(&p.tm_s0, q.w0.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, in / 64, rows_total, in / 32, in / 64,
                  tile_rows, CU_TENSOR_MAP_SWIZZLE_NONE));
  TF_TRY(make_map(&p.tm_b0, q.w0.biases, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, in / 64, rows_total, in / 32, in / 64,
                  tile_rows, CU_TENSOR_MAP_SWIZZLE_NONE));
  if (sw) {
    TF_TRY(make_map(&p.tm_q1, q.w1.q, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, in / 8, rows_total, in / 2, 8, tile_rows,
                    CU_TENSOR_MAP_SWIZZLE_NONE));
    TF_TRY(make_map(&p.tm_s1, q.w1.scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, in / 64, rows_total, in / 32,
                    in / 64, tile_rows, CU_TENSOR_MAP_SWIZZLE_NONE));
    TF_TRY(make_map(&p.tm_b1, q.w1.biases, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, in / 64, rows_total, in / 32,
                    in / 64, tile_rows, CU_TENSOR_MAP_SWIZZLE_NONE));
  }
  p.offsets = q.offsets;
  p.active = q.active;
  p.active_count = q.active_count;
  p.grouped = q.mode == QMM_GROUPED;
  p.row_blocks = (out + tile_rows - 1) / tile_rows;
  p.out = out;
  p.in = in;
  p.n = q.n;
  p.y = q.y;
  p.y_stride = q.y_stride;
  p.y_f16 = q.y_f16;
  p.residual = q.residual;
  p.residual_stride = q.residual_stride;
  // Token tile: about the tokens each weight matrix serves.
  const int64_t per_matrix = p.grouped ? (q.n + experts - 1) / experts : q.n;
  const int nt = per_matrix <= 24 ? 32 : per_matrix <= 64 ? 64 : 256;
  const int64_t token_tiles = p.grouped ? experts + q.n / nt + 1 : (q.n + nt - 1) / nt;
  const int64_t tiles_bound = token_tiles * p.row_blocks;
#define TF_TC_EPI(E)                                                                     \
  return q.act == TF_DTYPE_F16 ? launch_nt<__half, E>(p, q, nt, tiles_bound, s)          \
                               : launch_nt<__nv_bfloat16, E>(p, q, nt, tiles_bound, s);
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

// y[i] = f16(x[src(i)]) row by row, src(i) = perm ? perm[i] / div : i.  bf16
// -> f16 is exact for |x| in [2^-14, 65504]; beyond the f16 range the value
// would become inf, so such rows record error code 5.
template <typename Tin>
__global__ void gather_f16_kernel(const Tin* __restrict__ x, int64_t x_stride, const int32_t* __restrict__ perm,
                                  int div, int64_t rows, int width, __half* __restrict__ y) {
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
  *reinterpret_cast<uint4*>(y + row * width + 8 * c) = pack8<__half>(f);
}

tf_status launch_gather_f16(const void* x, int64_t x_stride, int act, const int32_t* perm, int div, int64_t rows,
                            int width, void* y, cudaStream_t s) {
  if (rows == 0) return TF_OK;
  if (width % 8) return set_error(TF_ERR_SHAPE, "gather_f16: width %d", width);
  const int64_t cpr = (width / 8 + 127) / 128;
  if (rows * cpr > 2147483647) return set_error(TF_ERR_UNSUPPORTED, "gather_f16: too many rows");
  const unsigned grid = (unsigned)(rows * cpr);
  if (act == TF_DTYPE_F16)
    gather_f16_kernel<__half><<<grid, 128, 0, s>>>((const __half*)x, x_stride, perm, div, rows, width, (__half*)y);
  else
    gather_f16_kernel<__nv_bfloat16><<<grid, 128, 0, s>>>((const __nv_bfloat16*)x, x_stride, perm, div, rows, width,
                                                          (__half*)y);
  return check_launch("gather_f16");
}

tf_status launch_bf16_to_f16(const void* x, int64_t n, void* y, cudaStream_t s) {
  if (n == 0) return TF_OK;
  if (n % 2048) return set_error(TF_ERR_SHAPE, "bf16_to_f16: count %lld not a multiple of 2048", (long long)n);
  return launch_gather_f16(x, 2048, TF_DTYPE_BF16, nullptr, 1, n / 2048, 2048, y, s);
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
