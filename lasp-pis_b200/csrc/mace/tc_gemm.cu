// FP32-accurate GEMM on the Blackwell tensor cores (tcgen05, kind::tf32, 3-term split).
//
//   C[z] (+)= A[z] * B      A: [M][K] fp32 row-major per batch z (node or edge features),
//                           B: given as two K-major tf32 planes Bhi/Blo [N][K] with
//                              B = Bhi + Blo (split once at model load).
// A needs no hi plane: an MMA of kind::tf32 reads the top 19 bits of each fp32 operand, so
// the loaded A tile itself acts as A_hi = trunc_tf32(a), and only
// A_lo = round_tf32(a - trunc_tf32(a)) is written beside it.  The remainder a - trunc(a) has
// the sign of a, so it is rounded (not left to the MMA's truncation) to keep the dropped part
// unbiased.  The tile product is accumulated in TMEM as A_hi*B_hi + A_lo*B_hi + A_hi*B_lo (the
// dropped parts are below 2^-21 relative and of either sign), so the result carries
// FP32-level error while the work runs on the tensor pipe.
//
// The tensor pipe adds products into its accumulator with truncation toward zero, which
// biases long accumulations coherently.  So the dominant A_hi*B_hi term is accumulated
// FRESH for every 32-wide K slab (4 MMAs) into one of two TMEM buffers and drained into
// FP32 registers with round-to-nearest adds (overlapping the next slab), while the two
// correction terms, 2^-11 smaller, accumulate over all of K in a per-tile correction
// buffer drained once at the end of the tile.
//
// Persistent: one CTA per SM walks the 128 x 128 output tiles (n fastest, so the CTAs that
// run together share A tiles in L2) with a continuous pipeline across tiles.  TMEM holds
// two slab buffers and two correction buffers (512 columns), so the MMAs of tile t+1 run
// while tile t is drained and stored.  CTA = 12 warps:
//   warp 0       TMA producer (A, Bhi, Blo per 32-wide K slab, SWIZZLE_128B, 3-stage ring)
//   warp 1       MMA issuer (one elected thread; UMMA 128 x 128 x 8)
//   warps 2..3   write A_lo beside the A tile in shared memory
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
#include <algorithm>
#include <climits>
#include <mutex>

namespace mace {
namespace {
using namespace tc;
constexpr int kBM = 128, kBN = 128, kBK = 32, kStages = 3;
constexpr int kTileBytes = kBM * kBK * 4;        // 16 KiB (A, A_lo, Bhi, Blo tiles are equal)
constexpr int kStageBytes = 4 * kTileBytes;      // A | A_lo | Bhi | Blo
constexpr int kBoxBytes = 32 * 32 * 4;           // one 32 x 32 output box (4 KiB)
constexpr int kStagingBytes = 8 * kBoxBytes;     // one box per drain warp
constexpr int kSmemBytes = 1024 /* align */ + kStages * kStageBytes + kStagingBytes + 128 /* barriers */;
static_assert(kSmemBytes + 64 <= 232448, "shared memory budget");
constexpr int kTmemCols = 4 * kBN; // hi*hi slab buffers 0/1, correction buffers 2/3 (512 columns)
constexpr int kThreads = 384, kDrainThreads = 256;
constexpr int kStatusGemmTimeout = 7;
constexpr int kMaxGemmProblems = 16, kMaxGemmSegments = 16;

// Instruction descriptor: D fp32, A/B tf32, both K-major, M = 128, N = 128.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (uint32_t(kBN >> 3) << 17) | (uint32_t(kBM >> 4) << 24);

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
  umma_tf32_desc(tmem_d, a, b, kIdesc, accumulate);
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
struct GemmSegment {
  CUtensorMap a, bhi, blo;
  int ktiles;
};
struct GemmProblem {
  CUtensorMap a, bhi, blo, c; // first K segment and the output
  TileGrid tg;
  int ktiles, kt0, accumulate, tile0; // total K tiles, the first segment's; first tile in the group
  int seg0, nseg;                     // further K segments
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
  uint64_t *bars = reinterpret_cast<uint64_t *>(staging + kStagingBytes);
  // bars: full[S] | ready[S] | empty[S] | tfull[2] | tfree[2] | cfull[2] | cfree[2] | done
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ int mma_done_issued; // whether the final commit to `done` was issued
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned full0 = smem_u32(bars), ready0 = full0 + 8 * kStages, empty0 = ready0 + 8 * kStages,
           tfull0 = empty0 + 8 * kStages, tfree0 = tfull0 + 16, cfull0 = tfree0 + 16, cfree0 = cfull0 + 16,
           done = cfree0 + 16;
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
      mbar_init(cfull0 + 8 * b, 1);
      mbar_init(cfree0 + 8 * b, kDrainThreads);
    }
    mbar_init(done, 1);
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
      for (int t = blockIdx.x; t < gg.tiles && ok; t += gridDim.x) {
        const GemmProblem &pr = gg.find(t, q);
        int n0, m0, z;
        pr.tg.coords(t - pr.tile0, n0, m0, z);
        for (int kt = 0; kt < pr.kt0; ++kt, ++g) {
          int s = g % kStages;
          if (g >= kStages && !(ok = mbar_wait(empty0 + 8 * s, ((g / kStages) - 1) & 1, &abort_flag)))
            break;
          unsigned base = smem_u32(smem + s * kStageBytes);
          mbar_expect_tx(full0 + 8 * s, 3 * kTileBytes);
          tma_load_3d(base, &pr.a, kt * kBK, m0, z, full0 + 8 * s);
          tma_load_2d(base + 2 * kTileBytes, &pr.bhi, kt * kBK, n0, full0 + 8 * s);
          tma_load_2d(base + 3 * kTileBytes, &pr.blo, kt * kBK, n0, full0 + 8 * s);
        }
        for (int sg = pr.seg0; sg < pr.seg0 + pr.nseg && ok; ++sg) {
          const GemmSegment &seg = gg.seg[sg];
          for (int kt = 0; kt < seg.ktiles; ++kt, ++g) {
            int s = g % kStages;
            if (g >= kStages && !(ok = mbar_wait(empty0 + 8 * s, ((g / kStages) - 1) & 1, &abort_flag)))
              break;
            unsigned base = smem_u32(smem + s * kStageBytes);
            mbar_expect_tx(full0 + 8 * s, 3 * kTileBytes);
            tma_load_3d(base, &seg.a, kt * kBK, m0, z, full0 + 8 * s);
            tma_load_2d(base + 2 * kTileBytes, &seg.bhi, kt * kBK, n0, full0 + 8 * s);
            tma_load_2d(base + 3 * kTileBytes, &seg.blo, kt * kBK, n0, full0 + 8 * s);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = true;
      int g = 0, i = 0, q = 0;
      for (int t = blockIdx.x; t < gg.tiles && ok; t += gridDim.x, ++i) {
        int ktiles = gg.find(t, q).ktiles, c = i & 1;
        if (i >= 2 && !(ok = mbar_wait(cfree0 + 8 * c, ((i >> 1) - 1) & 1, &abort_flag)))
          break;
        uint32_t corr = tmem + uint32_t((2 + c) * kBN);
        for (int kt = 0; kt < ktiles; ++kt, ++g) {
          int s = g % kStages, b = g & 1;
          if (!(ok = mbar_wait(ready0 + 8 * s, (g / kStages) & 1, &abort_flag)))
            break;
          if (g >= 2 && !(ok = mbar_wait(tfree0 + 8 * b, ((g >> 1) - 1) & 1, &abort_flag)))
            break;
          tc_fence_after();
          unsigned base = smem_u32(smem + s * kStageBytes);
#pragma unroll
          for (int j = 0; j < kBK / 8; ++j) {
            uint64_t a_hi = smem_desc(base + 32 * j), a_lo = smem_desc(base + kTileBytes + 32 * j);
            uint64_t b_hi = smem_desc(base + 2 * kTileBytes + 32 * j), b_lo = smem_desc(base + 3 * kTileBytes + 32 * j);
            umma_tf32(tmem + uint32_t(b * kBN), a_hi, b_hi, j ? 1u : 0u);
            umma_tf32(corr, a_lo, b_hi, (kt | j) ? 1u : 0u);
            umma_tf32(corr, a_hi, b_lo, 1u);
          }
          umma_commit(tfull0 + 8 * b);
          umma_commit(empty0 + 8 * s);
        }
        if (ok)
          umma_commit(cfull0 + 8 * c);
      }
      umma_commit(done);
      mma_done_issued = 1;
    }
  } else if (warp < 4) {
    // ---------------- A split: A_lo beside the tile (A_hi is the tile itself) ----------------
    int t = threadIdx.x - 64, g = 0, q = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < gg.tiles && ok; tile += gridDim.x)
      for (int kt = 0, ktiles = gg.find(tile, q).ktiles; kt < ktiles; ++kt, ++g) {
        int s = g % kStages;
        ok = mbar_wait(full0 + 8 * s, (g / kStages) & 1, &abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        const float4 *a = reinterpret_cast<const float4 *>(smem + s * kStageBytes);
        float4 *lo = reinterpret_cast<float4 *>(smem + s * kStageBytes + kTileBytes);
#pragma unroll
        for (int q = 0; q < kTileBytes / 16 / 64; ++q) {
          float4 v = a[t + 64 * q], l;
          l.x = tf32_hi(v.x - tf32_trunc(v.x)), l.y = tf32_hi(v.y - tf32_trunc(v.y));
          l.z = tf32_hi(v.z - tf32_trunc(v.z)), l.w = tf32_hi(v.w - tf32_trunc(v.w));
          lo[t + 64 * q] = l;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(ready0 + 8 * s);
      }
  } else {
    // ---------------- drain + store: lane = output row, 64 columns per warp ----------------
    int quarter = warp & 3, col0 = 64 * ((warp - 4) >> 2);
    uint32_t lane_addr = tmem + (uint32_t(quarter * 32) << 16) + uint32_t(col0);
    unsigned char *box = staging + (warp - 4) * kBoxBytes; // this warp's staging box
    bool ok = true;
    int g = 0, i = 0, q = 0;
    for (int t = blockIdx.x; t < gg.tiles && ok; t += gridDim.x, ++i) {
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
        tc_fence_after();
        uint32_t r0[32], r1[32];
        tmem_ld32_async(lane_addr + uint32_t(b * kBN), r0);
        tmem_ld32_async(lane_addr + uint32_t(b * kBN + 32), r1);
        tmem_wait_ld();
        tmem_anchor(r0);
        tmem_anchor(r1);
        tc_fence_before();
        mbar_arrive(tfree0 + 8 * b);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          acc[k] += __uint_as_float(r0[k]);
          acc[32 + k] += __uint_as_float(r1[k]);
        }
      }
      if (!ok)
        break;
      // Correction buffer: added while the two boxes are staged and stored.
      int c = i & 1;
      ok = mbar_wait(cfull0 + 8 * c, (i >> 1) & 1, &abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r0[32], r1[32];
      tmem_ld32_async(lane_addr + uint32_t((2 + c) * kBN), r0);
      tmem_ld32_async(lane_addr + uint32_t((2 + c) * kBN + 32), r1);
      tmem_wait_ld();
      tmem_anchor(r0);
      tmem_anchor(r1);
      tc_fence_before();
      mbar_arrive(cfree0 + 8 * c);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        // The previous store must have read the box before it is rewritten.
        if (lane == 0)
          bulk_wait_read();
        __syncwarp();
        // Row `lane` of the box: 16-byte chunk q at position q ^ (lane & 7) (SWIZZLE_128B).
        unsigned char *row = box + lane * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float *a = acc + 32 * j + 4 * q;
          const uint32_t *r = (j ? r1 : r0) + 4 * q;
          *reinterpret_cast<float4 *>(row + ((q ^ (lane & 7)) << 4)) =
              make_float4(a[0] + __uint_as_float(r[0]), a[1] + __uint_as_float(r[1]),
                          a[2] + __uint_as_float(r[2]), a[3] + __uint_as_float(r[3]));
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
  cuuint32_t box[3] = {kBK, cuuint32_t(box_rows), 1};
  cuuint32_t elem[3] = {1, 1, 1};
  CUresult r = encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, cuuint32_t(rank), const_cast<float *>(base), dims,
                         strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw lapis::Error("cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return map;
}
} // namespace

CUtensorMap tc_map_2d(const float *base, int cols, long long rows, int box_cols, int box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * 4) % 16 || box_cols * 4 > 128 || box_rows > 256)
    throw lapis::Error("tensor map operand is not 16-byte aligned or the box is too large");
  CUtensorMap map;
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(cols) * 4};
  cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(box_rows)};
  cuuint32_t elem[2] = {1, 1};
  CUresult r = encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box,
                         elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    throw lapis::Error("cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return map;
}

bool tc_gemm_supported(int N, int K) { return N % kBN == 0 && K % kBK == 0 && K >= kBK; }

namespace {
void check_problem(const GemmSpec &g) {
  if (!tc_gemm_supported(g.N, g.K))
    throw lapis::Error("tensor-core GEMM shape unsupported");
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
    CUtensorMap a = make_map(g.A, g.K, g.M, 3, g.batch, g.batch > 1 ? g.strideA : (long long)g.M * g.K);
    CUtensorMap bhi = make_map(g.Bhi, g.K, g.N, 2, 1, 0), blo = make_map(g.Blo, g.K, g.N, 2, 1, 0);
    if (!g.join) {
      p.a = a, p.bhi = bhi, p.blo = blo;
      p.kt0 = g.K / kBK;
    } else {
      GemmSegment &sg = gg.seg[ns++];
      sg.a = a, sg.bhi = bhi, sg.blo = blo;
      sg.ktiles = g.K / kBK;
      p.nseg += 1;
    }
    p.ktiles += g.K / kBK;
  }
  if (!n)
    return;
  gg.count = n;
  gg.tiles = int(tiles);
  int grid = int(std::min<long long>(tiles, sms));
  lapis::launch(tc_gemm_kernel, grid, kThreads, kSmemBytes, s, gg, status);
}
} // namespace

// C[z] (+)= A[z] * B  with B = Bhi + Blo given K-major ([N][K]); batch z = 0..batch-1.
void tc_gemm(cudaStream_t s, int M, int N, int K, int batch, const float *A, long long strideA, const float *Bhi,
             const float *Blo, float *C, int ldc, long long strideC, bool accumulate, int *status) {
  GemmSpec g{M, N, K, batch, A, strideA, Bhi, Blo, C, ldc, strideC, accumulate};
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
