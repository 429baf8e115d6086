// FP32-accurate GEMM on the Blackwell tensor cores (tcgen05, kind::f16, 3-term fp16 split).
//
//   C[z] (+)= A[z] * B      A: [M][K] fp32 row-major per batch z (node or edge features),
//                           B: given as two K-major fp16 planes Bhi/Blo [N][K] with
//                              B 2^eB = Bhi + Blo (split once at model load, split_f16).
// A may also arrive already split (GemmSpec::Ahi / Alo / Aexp, written by the kernel that
// produces it): the two fp16 planes are then loaded by TMA where the split would write them,
// and only the row exponents are read.  Otherwise each 128-row x 64-wide K slab of A is
// split in shared memory the same way, per row: with
// 2^e the power of two that brings the row's largest |a| into [2^14, 2^15),
// a 2^e = A_hi + A_lo, A_hi = round_fp16(a 2^e), A_lo = round_fp16(a 2^e - A_hi) (the
// remainder is exact in fp32).  Each pair carries 22 significant bits, and the scaling keeps
// every value of the row inside fp16's normal range down to 2^-17 of the row's largest.
// The slab product A_lo*B_hi + A_hi*B_lo + A_hi*B_hi (the dropped A_lo*B_lo is below 2^-22
// relative) runs on the fp16 tensor pipe, which has twice the tf32 rate.
//
// The tensor pipe adds products into its accumulator with truncation toward zero, which
// biases long accumulations coherently.  So every slab is accumulated FRESH in one of two
// TMEM buffers, the two correction terms first (their truncation is 2^-11 smaller), then the
// four A_hi*B_hi steps, and drained into FP32 registers with one fused multiply-add by
// 2^-(e + eB) (exact) and a round-to-nearest add, overlapping the next slab's MMAs.  The
// drain first moves each slab result one ulp away from zero, which cancels the measured mean
// shrinkage of a slab (one ulp on average) and leaves the product unbiased.
//
// Persistent: one CTA per SM walks the 128 x 128 output tiles (n fastest, so the CTAs that
// run together share A tiles in L2) with a continuous pipeline across tiles.  CTA = 12 warps:
//   warp 0       TMA producer: per slab the fp32 A tile (two 128 x 32 boxes) and the fp16
//                Bhi, Blo tiles (128 x 64 each), SWIZZLE_128B, 3-stage ring
//   warp 1       MMA issuer (one elected thread; UMMA 128 x 128 x 16)
//   warps 2..3   split A in place: a thread reads whole fp32 rows of the slab and writes the
//                row's A_hi over its first box and A_lo over its second (the fp16 K-major
//                SWIZZLE_128B layout has the same 128-byte rows), plus the row's exponent
//   warps 4..11  drain TMEM into FP32 registers: two warps per TMEM lane quadrant (lane =
//                output row), each owning 64 of the 128 columns with two 32-column loads in
//                flight; each writes its part of the tile as two 32 x 32 boxes staged
//                128B-swizzled in shared memory and stored by TMA tensor stores (fp32
//                add-reductions when accumulating); rows past M are clipped by the map
// Every mbarrier wait is bounded: on time-out the CTA records an error code in *status,
// stops issuing work, waits (bounded) for issued MMAs and frees its TMEM.
#include "../lapis/launch.cuh"
#include "model.hpp"
#include "tcgen05.cuh"
#include <cuda.h>
#include <cuda_fp16.h>
#include <algorithm>
#include <climits>
#include <mutex>

namespace mace {
namespace {
using namespace tc;
constexpr int kBM = 128, kBN = 128, kBK = 64, kStages = 3; // kBK: K per slab
constexpr int kTileBytes = kBM * kBK * 2;        // 16 KiB: one 128 x 64 fp16 operand tile
constexpr int kStageBytes = 4 * kTileBytes;      // fp32 A (then A_hi | A_lo) | Bhi | Blo
constexpr int kBoxBytes = 32 * 32 * 4;           // one 32 x 32 output box (4 KiB)
constexpr int kStagingBytes = 8 * kBoxBytes;     // one box per drain warp
// Row exponents e + eB of the last kExpSlots slabs (int16 per row).  The split of slab g runs
// only after the drain of slab g - 5 has released its TMEM buffer (TMA of g waits for the MMAs
// of g - 3, which wait for the drain of g - 5), so 6 slots are never overwritten early.
constexpr int kExpSlots = 6;
constexpr int kExpBytes = kExpSlots * kBM * 2;
constexpr int kSmemBytes = 1024 /* align */ + kStages * kStageBytes + kStagingBytes + kExpBytes + 256 /* barriers */;
static_assert(kSmemBytes + 64 <= 232448, "shared memory budget");
constexpr int kTmemCols = 2 * kBN; // two slab accumulators (256 columns)
constexpr int kThreads = 384, kDrainThreads = 256;
constexpr int kStatusGemmTimeout = 7;
constexpr int kMaxGemmProblems = 16, kMaxGemmSegments = 16;
constexpr uint32_t kIdesc = idesc_f16(kBM, kBN);

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
  umma_f16_desc(tmem_d, a, b, kIdesc, accumulate);
}

// Row exponent e: 2^e brings the row's largest magnitude m into [2^14, 2^15), with e and
// e + eB kept in [-126, 126] so that 2^e and 2^-(e + eB) are normal floats.
__device__ __forceinline__ int row_exponent(float m, int eb) {
  int ex = int(__float_as_uint(m) >> 23) & 0xff; // biased exponent (m >= 0)
  int e = ex ? 141 - ex : (m > 0.f ? 126 : 0);
  return min(max(e, max(-126, -126 - eb)), min(126, 126 - eb));
}
__device__ __forceinline__ float pow2(int e) { return __uint_as_float(uint32_t(127 + e) << 23); }
// A slab result one ulp larger in magnitude (zero stays zero).  The tensor pipe's
// accumulation truncates toward zero, and a slab's result measured 8.7e-8 smaller in mean
// relative magnitude than the exact product, independent of K: one ulp, which is 2^-23 / m
// of a result with mantissa m in [1, 2), 8.6e-8 on average over log-uniform mantissas.
// Without this step the shrinkage is coherent across every GEMM output and grows the virial
// error.
__device__ __forceinline__ uint32_t away_ulp(uint32_t bits) { return bits + ((bits << 1) != 0u); }

// Eight scaled values as fp16 hi and lo halves, packed for one 16-byte chunk of each plane
// (paired fp32 instructions: x = v sc, lo = x - float(hi), both exact).
__device__ __forceinline__ void split8(const float *v, float2 sc, uint4 &hi, uint4 &lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    float2 x = __fmul2_rn(make_float2(v[2 * p], v[2 * p + 1]), sc);
    __half2 hh = __float22half2_rn(x);
    float2 r = __ffma2_rn(__half22float2(hh), make_float2(-1.f, -1.f), x);
    __half2 ll = __float22half2_rn(r);
    h[p] = *reinterpret_cast<uint32_t *>(&hh);
    l[p] = *reinterpret_cast<uint32_t *>(&ll);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}

struct TileGrid {
  int nN, nM, tiles;
  __device__ void coords(int t, int &n0, int &m0, int &z) const {
    n0 = (t % nN) * kBN;
    int r = t / nN;
    m0 = (r % nM) * kBM;
    z = r / nM;
  }
};

// One launch runs a group of independent GEMMs (the paths of an equivariant linear) over
// their concatenated tile space, so short problems share one pipeline ramp and tail.  A
// problem's K range may be a concatenation of segments, each with its own A and B (paths
// that add into the same output block): C = sum_s A_s B_s accumulates inside the tile.
// A K segment's A operand: fp32 (split in the kernel), or given split (map a over A_hi, alo
// over A_lo, and the exponents aexp[z * xbatch + row * xrow + slab]).
struct SplitA {
  CUtensorMap alo;
  const int16_t *aexp;
  long long xbatch;
  int xrow, presplit;
};
struct GemmSegment {
  CUtensorMap a, bhi, blo;
  SplitA sa;
  int ktiles, eb; // K slabs; B's exponent eB
};
struct GemmProblem {
  CUtensorMap a, bhi, blo, c; // first K segment and the output
  SplitA sa;
  TileGrid tg;
  int M, ktiles, kt0, eb, accumulate, tile0; // rows; total K slabs, the first segment's and its eB; first tile
  int seg0, nseg;                            // further K segments
};
struct GemmGroup {
  GemmProblem p[kMaxGemmProblems];
  GemmSegment seg[kMaxGemmSegments];
  int count, tiles;
  // Problem of group tile t, advancing q (tiles are visited in increasing order).
  __device__ __forceinline__ const GemmProblem &find(int t, int &q) const {
    while (q + 1 < count && t >= p[q + 1].tile0)
      ++q;
    return p[q];
  }
};

__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ GemmGroup gg, int *status) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *staging = smem + kStages * kStageBytes;
  int16_t *exps = reinterpret_cast<int16_t *>(staging + kStagingBytes); // [kExpSlots][kBM]
  uint64_t *bars = reinterpret_cast<uint64_t *>(staging + kStagingBytes + kExpBytes);
  // bars: full[S] | ready[S] | empty[S] | tfull[2] | tfree[2] | done | xfull[kExpSlots]
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ int mma_done_issued; // whether the final commit to `done` was issued
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned full0 = smem_u32(bars), ready0 = full0 + 8 * kStages, empty0 = ready0 + 8 * kStages,
           tfull0 = empty0 + 8 * kStages, tfree0 = tfull0 + 16, done = tfree0 + 16, xfull0 = done + 8;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mma_done_issued = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(ready0 + 8 * s, 64);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tfree0 + 8 * b, kDrainThreads);
    }
    mbar_init(done, 1);
    for (int x = 0; x < kExpSlots; ++x)
      mbar_init(xfull0 + 8 * x, 64);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int g = 0, q = 0;
      bool ok = true;
      auto load = [&](const CUtensorMap *a, const SplitA &sa, const CUtensorMap *bhi, const CUtensorMap *blo, int kt,
                      int n0, int m0, int z) {
        int s = g % kStages;
        if (g >= kStages && !(ok = mbar_wait(empty0 + 8 * s, ((g / kStages) - 1) & 1, &abort_flag)))
          return;
        unsigned base = smem_u32(smem + s * kStageBytes), full = full0 + 8 * s;
        mbar_expect_tx(full, kStageBytes);
        if (sa.presplit) { // A_hi and A_lo as they will sit after the split
          tma_load_3d(base, a, kt * kBK, m0, z, full);
          tma_load_3d(base + kTileBytes, &sa.alo, kt * kBK, m0, z, full);
        } else { // the two fp32 boxes
          tma_load_3d(base, a, kt * kBK, m0, z, full);
          tma_load_3d(base + kTileBytes, a, kt * kBK + 32, m0, z, full);
        }
        tma_load_2d(base + 2 * kTileBytes, bhi, kt * kBK, n0, full);
        tma_load_2d(base + 3 * kTileBytes, blo, kt * kBK, n0, full);
        ++g;
      };
      for (int t = blockIdx.x; t < gg.tiles && ok; t += gridDim.x) {
        const GemmProblem &pr = gg.find(t, q);
        int n0, m0, z;
        pr.tg.coords(t - pr.tile0, n0, m0, z);
        for (int kt = 0; kt < pr.kt0 && ok; ++kt)
          load(&pr.a, pr.sa, &pr.bhi, &pr.blo, kt, n0, m0, z);
        for (int sg = pr.seg0; sg < pr.seg0 + pr.nseg && ok; ++sg)
          for (int kt = 0; kt < gg.seg[sg].ktiles && ok; ++kt)
            load(&gg.seg[sg].a, gg.seg[sg].sa, &gg.seg[sg].bhi, &gg.seg[sg].blo, kt, n0, m0, z);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = true;
      int g = 0, q = 0;
      for (int t = blockIdx.x; t < gg.tiles && ok; t += gridDim.x) {
        int ktiles = gg.find(t, q).ktiles;
        for (int kt = 0; kt < ktiles; ++kt, ++g) {
          int s = g % kStages, b = g & 1;
          if (!(ok = mbar_wait(ready0 + 8 * s, (g / kStages) & 1, &abort_flag)))
            break;
          if (g >= 2 && !(ok = mbar_wait(tfree0 + 8 * b, ((g >> 1) - 1) & 1, &abort_flag)))
            break;
          tc_fence_after();
          unsigned base = smem_u32(smem + s * kStageBytes);
          uint32_t d = tmem + uint32_t(b * kBN);
          // 16-wide K steps are 32 bytes apart inside the 128-byte swizzled rows.
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j) {
            umma(d, smem_desc(base + kTileBytes + 32 * j), smem_desc(base + 2 * kTileBytes + 32 * j), j ? 1u : 0u);
            umma(d, smem_desc(base + 32 * j), smem_desc(base + 3 * kTileBytes + 32 * j), 1u);
          }
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j)
            umma(d, smem_desc(base + 32 * j), smem_desc(base + 2 * kTileBytes + 32 * j), 1u);
          umma_commit(tfull0 + 8 * b);
          umma_commit(empty0 + 8 * s);
        }
      }
      umma_commit(done);
      mma_done_issued = 1;
    }
  } else if (warp < 4) {
    // ---------------- A split, in place: rows t and t + 64 of every slab ----------------
    int t = threadIdx.x - 64, g = 0, q = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < gg.tiles && ok; tile += gridDim.x) {
      const GemmProblem &pr = gg.find(tile, q);
      int n0, m0, z;
      pr.tg.coords(tile - pr.tile0, n0, m0, z);
      int sg = pr.seg0 - 1, left = pr.kt0, eb = pr.eb, slabs = pr.kt0;
      const SplitA *sa = &pr.sa;
      for (int kt = 0; kt < pr.ktiles; ++kt, ++g) {
        while (!left) { // the slab's K segment, its B exponent and its A
          ++sg;
          left = slabs = gg.seg[sg].ktiles;
          eb = gg.seg[sg].eb;
          sa = &gg.seg[sg].sa;
        }
        int ks = slabs - left; // slab within the segment
        --left;
        // A split operand's exponents come from global memory: load them before waiting for the
        // slab, so the load overlaps the wait.
        int pe[2] = {0, 0};
        if (sa->presplit) {
#pragma unroll
          for (int h = 0; h < 2; ++h)
            if (m0 + t + 64 * h < pr.M)
              pe[h] = sa->aexp[z * sa->xbatch + (long long)(m0 + t + 64 * h) * sa->xrow + ks];
        }
        int s = g % kStages;
        ok = mbar_wait(full0 + 8 * s, (g / kStages) & 1, &abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        unsigned char *st = smem + s * kStageBytes;
        int16_t *ex = exps + (g % kExpSlots) * kBM;
        if (sa->presplit) { // A arrived split: only its exponents, offset by eB
#pragma unroll
          for (int h = 0; h < 2; ++h)
            ex[t + 64 * h] = int16_t(min(max(pe[h] + eb, -126), 126));
        } else {
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            int r = t + 64 * h, sw = r & 7;
            unsigned char *ra = st + r * 128, *rb = st + kTileBytes + r * 128; // row r of each box
            float v[64];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              float4 x = *reinterpret_cast<const float4 *>(ra + ((c ^ sw) << 4));
              float4 y = *reinterpret_cast<const float4 *>(rb + ((c ^ sw) << 4));
              v[4 * c] = x.x, v[4 * c + 1] = x.y, v[4 * c + 2] = x.z, v[4 * c + 3] = x.w;
              v[32 + 4 * c] = y.x, v[33 + 4 * c] = y.y, v[34 + 4 * c] = y.z, v[35 + 4 * c] = y.w;
            }
            // Row maximum as an 8-way tree (short dependency chains).
            float mx[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
              mx[j] = fabsf(v[j]);
#pragma unroll
            for (int k = 8; k < 64; ++k)
              mx[k & 7] = fmaxf(mx[k & 7], fabsf(v[k]));
#pragma unroll
            for (int w = 4; w; w >>= 1)
#pragma unroll
              for (int j = 0; j < w; ++j)
                mx[j] = fmaxf(mx[j], mx[j + w]);
            int e = row_exponent(mx[0], eb);
            float2 sc = make_float2(pow2(e), pow2(e));
            // fp16 chunk c holds elements 8c .. 8c + 7 of the row: A_hi over the first box,
            // A_lo over the second, at the same swizzled positions.
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint4 hi, lo;
              split8(v + 8 * c, sc, hi, lo);
              *reinterpret_cast<uint4 *>(ra + ((c ^ sw) << 4)) = hi;
              *reinterpret_cast<uint4 *>(rb + ((c ^ sw) << 4)) = lo;
            }
            ex[r] = int16_t(e + eb);
          }
        }
        mbar_arrive(xfull0 + 8 * (g % kExpSlots)); // the exponents, for the drain
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(ready0 + 8 * s);
      }
    }
  } else {
    // ---------------- drain + store: lane = output row, 64 columns per warp ----------------
    int quarter = warp & 3, col0 = 64 * ((warp - 4) >> 2), row = 32 * quarter + lane;
    uint32_t lane_addr = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(col0);
    unsigned char *box = staging + (warp - 4) * kBoxBytes; // this warp's staging box
    bool ok = true;
    int g = 0, q = 0;
    for (int t = blockIdx.x; t < gg.tiles && ok; t += gridDim.x) {
      const GemmProblem &pr = gg.find(t, q);
      int n0, m0, z, ktiles = pr.ktiles;
      pr.tg.coords(t - pr.tile0, n0, m0, z);
      float acc[64];
#pragma unroll
      for (int c = 0; c < 64; ++c)
        acc[c] = 0.f;
      for (int kt = 0; kt < ktiles; ++kt, ++g) {
        int b = g & 1;
        ok = mbar_wait(tfull0 + 8 * b, (g >> 1) & 1, &abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        int x = g % kExpSlots;
        ok = mbar_wait(xfull0 + 8 * x, (g / kExpSlots) & 1, &abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r0[32], r1[32];
        tmem_ld32_async(lane_addr + uint32_t(b * kBN), r0);
        tmem_ld32_async(lane_addr + uint32_t(b * kBN + 32), r1);
        float inv = pow2(-int(exps[x * kBM + row]));
        tmem_wait_ld();
        tmem_anchor(r0);
        tmem_anchor(r1);
        tc_fence_before();
        mbar_arrive(tfree0 + 8 * b);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          acc[k] = fmaf(__uint_as_float(away_ulp(r0[k])), inv, acc[k]);
          acc[32 + k] = fmaf(__uint_as_float(away_ulp(r1[k])), inv, acc[32 + k]);
        }
      }
      if (!ok)
        break;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        // The previous store must have read the box before it is rewritten.
        if (lane == 0)
          bulk_wait_read();
        __syncwarp();
        // Row `lane` of the box: 16-byte chunk q at position q ^ (lane & 7) (SWIZZLE_128B).
        unsigned char *rowp = box + lane * 128;
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4) {
          const float *a = acc + 32 * j + 4 * q4;
          *reinterpret_cast<float4 *>(rowp + ((q4 ^ (lane & 7)) << 4)) = make_float4(a[0], a[1], a[2], a[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          int x = n0 + col0 + 32 * j, y = m0 + 32 * quarter;
          if (pr.accumulate)
            tma_add_3d(&pr.c, smem_u32(box), x, y, z);
          else
            tma_store_3d(&pr.c, smem_u32(box), x, y, z);
          bulk_commit();
        }
      }
    }
    if (lane == 0)
      bulk_wait();
  }
  tc_fence_before();
  __syncthreads();
  if (abort_flag && threadIdx.x == 0)
    atomicCAS(status, 0, kStatusGemmTimeout);
  if (warp == 1) {
    if (abort_flag && mma_done_issued) {
      // Drain: the final commit was issued; wait (bounded) for the MMAs before freeing TMEM.
      long long start = clock64();
      while (!mbar_try(done, 0) && clock64() - start < kWaitCycles) {
      }
    }
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encoder() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  });
  if (!fn)
    throw lapis::Error("cuTensorMapEncodeTiled is unavailable");
  return fn;
}

// Tensor map over `rows` x `cols` fp32 (row stride `ld` elements, default cols) [x `batch`
// planes when rank 3], box 32 (cols) x `box_rows` (rows) [x 1], SWIZZLE_128B.
CUtensorMap make_map(const float *base, int cols, int rows, int rank, int batch, long long batch_stride,
                     int ld = 0, int box_rows = kBM) {
  if (!ld)
    ld = cols;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 4) % 16 || (batch_stride * 4) % 16)
    throw lapis::Error("tensor-core GEMM operand is not 16-byte aligned");
  CUtensorMap map;
  cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(rows), cuuint64_t(batch)};
  cuuint64_t strides[2] = {cuuint64_t(ld) * 4, cuuint64_t(batch_stride) * 4};
  cuuint32_t box[3] = {32, cuuint32_t(box_rows), 1};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, cuuint32_t(rank), const_cast<float *>(base), dims,
                         strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw lapis::Error("cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return map;
}

// Tensor map over a split A plane [batch][M][K] fp16 (batch stride in elements), box 64 (K) x
// 128 (rows) x 1, SWIZZLE_128B: the layout the in-kernel split writes.
CUtensorMap make_map_f16_a(const uint16_t *base, int K, int M, int batch, long long batch_stride) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (K * 2) % 16 || (batch_stride * 2) % 16)
    throw lapis::Error("tensor-core GEMM split operand is not 16-byte aligned");
  CUtensorMap map;
  cuuint64_t dims[3] = {cuuint64_t(K), cuuint64_t(M), cuuint64_t(batch)};
  cuuint64_t strides[2] = {cuuint64_t(K) * 2, cuuint64_t(batch_stride) * 2};
  cuuint32_t box[3] = {kBK, kBM, 1};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<uint16_t *>(base), dims, strides, box,
                         elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw lapis::Error("cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return map;
}

// Tensor map over an fp16 B plane [N][K], box 64 (K) x 128 (N), SWIZZLE_128B.
CUtensorMap make_map_f16(const uint16_t *base, int K, int N) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (K * 2) % 16)
    throw lapis::Error("tensor-core GEMM operand is not 16-byte aligned");
  CUtensorMap map;
  cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(N)};
  cuuint64_t strides[1] = {cuuint64_t(K) * 2};
  cuuint32_t box[2] = {kBK, kBN};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t *>(base), dims, strides, box,
                         elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw lapis::Error("cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return map;
}
} // namespace

// K in multiples of 32: the last slab of a K = 32 mod 64 problem reads zeros past K.
bool tc_gemm_supported(int N, int K) { return N % kBN == 0 && K % 32 == 0 && K >= 32; }

namespace {
void check_problem(const GemmSpec &g) {
  if (!tc_gemm_supported(g.N, g.K))
    throw lapis::Error("tensor-core GEMM shape unsupported");
  if (g.Ahi && (g.K % kBK || !g.Alo || !g.Aexp))
    throw lapis::Error("tensor-core GEMM split operand needs K a multiple of 64, both planes and exponents");
  if ((reinterpret_cast<uintptr_t>(g.C) & 15) || g.ldc % 4 || (g.batch > 1 && g.strideC % 4))
    throw lapis::Error("tensor-core GEMM output is not 16-byte aligned");
}

void launch_group(cudaStream_t s, const GemmSpec *specs, int count, int *status) {
  static thread_local int configured_device = -1, sms = 148;
  int device = 0;
  lapis::check(cudaGetDevice(&device));
  if (configured_device != device) {
    lapis::check(cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    lapis::check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    configured_device = device;
  }
  GemmGroup gg{};
  long long tiles = 0;
  int n = 0, ns = 0;
  for (int k = 0; k < count; ++k) {
    const GemmSpec &g = specs[k];
    if (!g.M || !g.batch)
      continue;
    if (!g.join) {
      GemmProblem &p = gg.p[n++];
      // C as [batch][M][ldc], written in 32 x 32 boxes over its first N columns.
      p.c = make_map(g.C, g.N, g.M, 3, g.batch, g.batch > 1 ? g.strideC : (long long)g.M * g.ldc, g.ldc, 32);
      p.tg = TileGrid{g.N / kBN, (g.M + kBM - 1) / kBM, 0};
      long long pt = (long long)p.tg.nN * p.tg.nM * g.batch;
      p.tg.tiles = int(std::min<long long>(pt, INT_MAX));
      p.accumulate = g.accumulate;
      p.tile0 = int(std::min<long long>(tiles, INT_MAX));
      p.seg0 = ns;
      tiles += pt;
      if (tiles > INT_MAX)
        throw lapis::Error("tensor-core GEMM has too many tiles");
    }
    GemmProblem &p = gg.p[n - 1];
    // A as [batch][M][K] (always a rank-3 map: the kernel issues 3D loads); B as [N][K].
    long long sA = g.batch > 1 ? g.strideA : (long long)g.M * g.K;
    CUtensorMap a;
    SplitA sa{};
    if (g.Ahi) {
      a = make_map_f16_a(g.Ahi, g.K, g.M, g.batch, sA);
      sa.alo = make_map_f16_a(g.Alo, g.K, g.M, g.batch, sA);
      sa.aexp = g.Aexp;
      sa.xbatch = g.strideAexp;
      sa.xrow = g.K / kBK;
      sa.presplit = 1;
    } else {
      a = make_map(g.A, g.K, g.M, 3, g.batch, sA);
    }
    CUtensorMap bhi = make_map_f16(g.B.hi, g.K, g.N), blo = make_map_f16(g.B.lo, g.K, g.N);
    int slabs = (g.K + kBK - 1) / kBK;
    if (!g.join) {
      p.a = a, p.bhi = bhi, p.blo = blo, p.sa = sa;
      p.M = g.M;
      p.kt0 = slabs;
      p.eb = g.B.exp;
    } else {
      GemmSegment &sg = gg.seg[ns++];
      sg.a = a, sg.bhi = bhi, sg.blo = blo, sg.sa = sa;
      sg.ktiles = slabs;
      sg.eb = g.B.exp;
      p.nseg += 1;
    }
    p.ktiles += slabs;
  }
  if (!n)
    return;
  gg.count = n;
  gg.tiles = int(tiles);
  int grid = int(std::min<long long>(tiles, sms));
  lapis::launch(tc_gemm_kernel, grid, kThreads, kSmemBytes, s, gg, status);
}
} // namespace

// C[z] (+)= A[z] * B  with B given as its fp16 split (K-major, [N][K]); batch z = 0..batch-1.
void tc_gemm(cudaStream_t s, int M, int N, int K, int batch, const float *A, long long strideA, const TCMatrix &B,
             float *C, int ldc, long long strideC, bool accumulate, int *status) {
  GemmSpec g{M, N, K, batch, A, strideA, B, C, ldc, strideC, accumulate};
  tc_gemm_group(s, &g, 1, status);
}

void tc_gemm_group(cudaStream_t s, const GemmSpec *specs, int count, int *status) {
  for (int k = 0; k < count; ++k) {
    const GemmSpec &g = specs[k];
    if (!g.M || !g.batch)
      continue;
    check_problem(g);
    if (g.join && (k == 0 || specs[k - 1].M != g.M || specs[k - 1].N != g.N || specs[k - 1].batch != g.batch ||
                   specs[k - 1].C != g.C || specs[k - 1].ldc != g.ldc || specs[k - 1].strideC != g.strideC ||
                   specs[k - 1].accumulate != g.accumulate))
      throw lapis::Error("tensor-core GEMM segment does not match its problem");
  }
  // Launches of at most kMaxGemmProblems problems and kMaxGemmSegments further segments; a
  // problem's segments stay in one launch.
  for (int k = 0; k < count;) {
    int end = k, problems = 0, segments = 0;
    while (end < count) {
      int e = end + 1;
      while (e < count && specs[e].join)
        ++e;
      if (e - end - 1 > kMaxGemmSegments)
        throw lapis::Error("tensor-core GEMM problem has too many segments");
      if (problems + 1 > kMaxGemmProblems || segments + (e - end - 1) > kMaxGemmSegments)
        break;
      ++problems;
      segments += e - end - 1;
      end = e;
    }
    launch_group(s, specs + k, end - k, status);
    k = end;
  }
}
} // namespace mace
