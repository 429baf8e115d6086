// FP32-accurate GEMM on the Blackwell tensor cores (tcgen05, kind::tf32, 3-term split).
//
//   C[z] (+)= A[z] * B      A: [M][K] fp32 row-major per batch z (node or edge features),
//                           B: given as two K-major tf32 planes Bhi/Blo [N][K] with
//                              B = Bhi + Blo (split once at model load).
// Each A tile is split on the fly into hi = round_tf32(a) and lo = a - hi, and the tile
// product is accumulated in TMEM as  A_hi*B_hi + A_lo*B_hi + A_hi*B_lo  (the dropped
// A_lo*B_lo term is below 2^-22 relative), so the result carries FP32-level error while the
// work runs on the tensor pipe.
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
// while tile t is drained and stored.  CTA = 8 warps (two per SM sub-partition, so the
// drain warps may hold a full 128-column row of FP32 accumulators):
//   warp 0      TMA producer (A, Bhi, Blo per 32-wide K slab, SWIZZLE_128B, 2-stage ring)
//   warp 1      MMA issuer (one elected thread; UMMA 128 x 128 x 8)
//   warps 2..5  drain TMEM (lane = output row) into FP32 registers, stage the row in
//               shared memory and write it with one bulk copy per row (a bulk fp32 add
//               into C when accumulating); rows past M are skipped
//   warps 6..7  split A into hi/lo in shared memory
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
constexpr int kBM = 128, kBN = 128, kBK = 32, kStages = 2;
constexpr int kTileBytes = kBM * kBK * 4;        // 16 KiB (A, A_lo, Bhi, Blo tiles are equal)
constexpr int kStageBytes = 4 * kTileBytes;      // A | A_lo | Bhi | Blo
constexpr int kRowStage = (kBN + 4) * 4;         // one staged output row, padded (528 B)
constexpr int kStagingBytes = kBM * kRowStage;   // 66 KiB
constexpr int kSmemBytes = 1024 /* align */ + kStages * kStageBytes + kStagingBytes + 256 /* barriers */;
constexpr int kTmemCols = 4 * kBN; // hi*hi slab buffers 0/1, correction buffers 2/3 (512 columns)
constexpr int kThreads = 256;
constexpr int kStatusGemmTimeout = 7;

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

__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmBhi,
                   const __grid_constant__ CUtensorMap tmBlo, float *C, int ldc, long long strideC, int M,
                   TileGrid tg, int K, int accumulate, int *status) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *staging = smem + kStages * kStageBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(staging + kStagingBytes);
  // bars: full[S] | ready[S] | empty[S] | tfull[2] | tfree[2] | cfull[2] | cfree[2] | done
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ int mma_done_issued; // whether the final commit to `done` was issued
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int ktiles = K / kBK;
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
      mbar_init(tfree0 + 8 * b, 128);
      mbar_init(cfull0 + 8 * b, 1);
      mbar_init(cfree0 + 8 * b, 128);
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
      int g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tg.tiles && ok; t += gridDim.x) {
        int n0, m0, z;
        tg.coords(t, n0, m0, z);
        for (int kt = 0; kt < ktiles; ++kt, ++g) {
          int s = g % kStages;
          if (g >= kStages && !(ok = mbar_wait(empty0 + 8 * s, ((g / kStages) - 1) & 1, &abort_flag)))
            break;
          unsigned base = smem_u32(smem + s * kStageBytes);
          mbar_expect_tx(full0 + 8 * s, 3 * kTileBytes);
          tma_load_3d(base, &tmA, kt * kBK, m0, z, full0 + 8 * s);
          tma_load_2d(base + 2 * kTileBytes, &tmBhi, kt * kBK, n0, full0 + 8 * s);
          tma_load_2d(base + 3 * kTileBytes, &tmBlo, kt * kBK, n0, full0 + 8 * s);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      bool ok = true;
      int g = 0, i = 0;
      for (int t = blockIdx.x; t < tg.tiles && ok; t += gridDim.x, ++i) {
        int c = i & 1;
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
  } else if (warp >= 6) {
    // ---------------- A split: hi in place, lo beside it ----------------
    int t = threadIdx.x - 192, g = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tg.tiles && ok; tile += gridDim.x)
      for (int kt = 0; kt < ktiles; ++kt, ++g) {
        int s = g % kStages;
        ok = mbar_wait(full0 + 8 * s, (g / kStages) & 1, &abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          ok = false;
          break;
        }
        float4 *a = reinterpret_cast<float4 *>(smem + s * kStageBytes);
        float4 *lo = reinterpret_cast<float4 *>(smem + s * kStageBytes + kTileBytes);
#pragma unroll
        for (int q = 0; q < kTileBytes / 16 / 64; ++q) {
          float4 v = a[t + 64 * q], h, l;
          h.x = tf32_hi(v.x), h.y = tf32_hi(v.y), h.z = tf32_hi(v.z), h.w = tf32_hi(v.w);
          l.x = v.x - h.x, l.y = v.y - h.y, l.z = v.z - h.z, l.w = v.w - h.w;
          a[t + 64 * q] = h;
          lo[t + 64 * q] = l;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(ready0 + 8 * s);
      }
  } else {
    // ---------------- drain + store: lane = output row ----------------
    int quarter = warp & 3, row_in_tile = quarter * 32 + lane;
    uint32_t lane_addr = tmem + (uint32_t(quarter * 32) << 16);
    unsigned char *my_row = staging + row_in_tile * kRowStage;
    bool ok = true;
    int g = 0, i = 0;
    for (int t = blockIdx.x; t < tg.tiles && ok; t += gridDim.x, ++i) {
      int n0, m0, z;
      tg.coords(t, n0, m0, z);
      float acc[kBN];
#pragma unroll
      for (int c = 0; c < kBN; ++c)
        acc[c] = 0.f;
      auto drain = [&](uint32_t col, uint32_t full, int parity, uint32_t release) {
        bool go = mbar_wait(full, parity, &abort_flag);
        if (!__all_sync(0xffffffffu, go))
          return false;
        tc_fence_after();
#pragma unroll
        for (int c0 = 0; c0 < kBN; c0 += 32) {
          float v[32];
          tmem_ld32(lane_addr + col + uint32_t(c0), v);
#pragma unroll
          for (int k = 0; k < 32; ++k)
            acc[c0 + k] += v[k];
        }
        tc_fence_before();
        mbar_arrive(release);
        return true;
      };
      for (int kt = 0; kt < ktiles && ok; ++kt, ++g) {
        int b = g & 1;
        ok = drain(uint32_t(b * kBN), tfull0 + 8 * b, (g >> 1) & 1, tfree0 + 8 * b);
      }
      int c = i & 1;
      if (ok)
        ok = drain(uint32_t((2 + c) * kBN), cfull0 + 8 * c, (i >> 1) & 1, cfree0 + 8 * c);
      if (!ok)
        break;
      // The previous tile's copy must have read this row's staging before it is rewritten.
      bulk_wait_read();
      float4 *dst = reinterpret_cast<float4 *>(my_row);
#pragma unroll
      for (int q = 0; q < kBN / 4; ++q)
        dst[q] = make_float4(acc[4 * q], acc[4 * q + 1], acc[4 * q + 2], acc[4 * q + 3]);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      int row = m0 + row_in_tile;
      if (row < M) {
        float *out = C + z * strideC + size_t(row) * ldc + n0;
        if (accumulate)
          bulk_add_f32(out, smem_u32(my_row), kBN * 4);
        else
          bulk_store(out, smem_u32(my_row), kBN * 4);
        bulk_commit();
      }
    }
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

// Tensor map over `rows` x `cols` fp32 (row-major, ld = cols) [x `batch` planes when rank 3],
// box 32 (cols) x 128 (rows) [x 1].
CUtensorMap make_map(const float *base, int cols, int rows, int rank, int batch, long long batch_stride) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * 4) % 16 || (batch_stride * 4) % 16)
    throw lapis::Error("tensor-core GEMM operand is not 16-byte aligned");
  CUtensorMap map;
  cuuint64_t dims[3] = {cuuint64_t(cols), cuuint64_t(rows), cuuint64_t(batch)};
  cuuint64_t strides[2] = {cuuint64_t(cols) * 4, cuuint64_t(batch_stride) * 4};
  cuuint32_t box[3] = {kBK, kBM, 1};
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

// C[z] (+)= A[z] * B  with B = Bhi + Blo given K-major ([N][K]); batch z = 0..batch-1.
void tc_gemm(cudaStream_t s, int M, int N, int K, int batch, const float *A, long long strideA, const float *Bhi,
             const float *Blo, float *C, int ldc, long long strideC, bool accumulate, int *status) {
  if (!M || !batch)
    return;
  if (!tc_gemm_supported(N, K))
    throw lapis::Error("tensor-core GEMM shape unsupported");
  if ((reinterpret_cast<uintptr_t>(C) & 15) || ldc % 4 || (batch > 1 && strideC % 4))
    throw lapis::Error("tensor-core GEMM output is not 16-byte aligned");
  // A as [batch][M][K] (always a rank-3 map: the kernel issues 3D loads); B as [N][K].
  CUtensorMap ma = make_map(A, K, M, 3, batch, batch > 1 ? strideA : (long long)M * K);
  CUtensorMap mh = make_map(Bhi, K, N, 2, 1, 0), ml = make_map(Blo, K, N, 2, 1, 0);
  static thread_local int configured_device = -1, sms = 148;
  int device = 0;
  lapis::check(cudaGetDevice(&device));
  if (configured_device != device) {
    lapis::check(cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
    lapis::check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    configured_device = device;
  }
  TileGrid tg{N / kBN, (M + kBM - 1) / kBM, 0};
  long long tiles = (long long)tg.nN * tg.nM * batch;
  if (tiles > INT_MAX)
    throw lapis::Error("tensor-core GEMM has too many tiles");
  tg.tiles = int(tiles);
  int grid = int(std::min<long long>(tiles, sms));
  lapis::launch(tc_gemm_kernel, grid, kThreads, kSmemBytes, s, ma, mh, ml, C, ldc, strideC, M, tg, K,
                int(accumulate), status);
}
} // namespace mace
