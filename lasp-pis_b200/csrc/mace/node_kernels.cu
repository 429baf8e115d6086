// MH1 node kernels for B200: equivariant linears, normalisation + gate, the symmetric
// contraction (cubic product basis) and small elementwise ops.
//
// Reference semantics (LipidL/LASP-PIS mace/src/mh1.cu):
//   linear()                  85-106   per path and component Y (+)= X W, or X_grad += Y_grad W^T
//   embed_kernel              107-120  species embedding (unknown element -> status 2)
//   normalize_kernel          121-128  pre = raw / (alpha + beta * density) + res
//   gate_kernel<false/true>   129-159  SiLU scalars, sigmoid-gated l = 1..3 blocks, and the VJP
//   norm_backward             160-176  VJP of the density normalisation
//   product_kernel            177-214  sparse cubic polynomial per channel and its VJP
//   read_act                  225-235  readout SiLU and its VJP
// Normalisation and gating are fused into one pass (forward) and one pass with the
// normalisation VJP (backward); the reference launches them separately.
#include "model.hpp"
#include "product_table.h"
#include "tcgen05.cuh"
#include <type_traits>
#include "../lapis/launch.cuh"
#include <cstdlib>
#include <cuda_fp16.h>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

namespace mace {
namespace {
__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + expf(-x)); }

// ---------------- FP32 GEMM: C[z] += A[z] * B  (B optionally read transposed) ----------------
constexpr int BM = 64, BN = 64, BK = 16;
template <bool TransB>
__global__ void __launch_bounds__(256) gemm_kernel(int M, int N, int K, const float *__restrict__ A, int lda,
                                                   long long sA, const float *__restrict__ B, int ldb,
                                                   float *__restrict__ C, int ldc, long long sC) {
  __shared__ __align__(16) float As[BK][BM + 4];
  __shared__ __align__(16) float Bs[BK][BN + 4];
  A += blockIdx.z * sA;
  C += blockIdx.z * sC;
  int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      int idx = tid + 256 * q, r = idx >> 4, kk = idx & 15, gm = m0 + r, gk = k0 + kk;
      As[kk][r] = (gm < M && gk < K) ? A[size_t(gm) * lda + gk] : 0.f;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      int idx = tid + 256 * q;
      if (!TransB) {
        int kk = idx >> 6, nn = idx & 63, gk = k0 + kk, gn = n0 + nn;
        Bs[kk][nn] = (gk < K && gn < N) ? B[size_t(gk) * ldb + gn] : 0.f;
      } else {
        int nn = idx >> 4, kk = idx & 15, gk = k0 + kk, gn = n0 + nn;
        Bs[kk][nn] = (gk < K && gn < N) ? B[size_t(gn) * ldb + gk] : 0.f;
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float4 a = *reinterpret_cast<const float4 *>(&As[kk][ty * 4]);
      float4 b = *reinterpret_cast<const float4 *>(&Bs[kk][tx * 4]);
      float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c)
          acc[r][c] = fmaf(av[r], bv[c], acc[r][c]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    int gm = m0 + ty * 4 + r;
    if (gm >= M)
      continue;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      int gn = n0 + tx * 4 + c;
      if (gn < N)
        C[size_t(gm) * ldc + gn] += acc[r][c];
    }
  }
}

// ---------------- skinny FP32 GEMM for N <= 16 (the readouts): C[z] += A[z] * B ----------------
// Warp per row.  The row of A is read in coalesced float4 chunks of 128 (lane = 4 columns),
// B sits in shared memory transposed and zero-padded ([NP][KP], NP = N rounded up to a power
// of two), so each lane forms NP partial dot products; a halving exchange then leaves lane l
// with the row total of column l (NP - 1 + 5 - log2(NP) shuffles).  Needs K, lda multiples of
// 4 and a 16-byte aligned A.
constexpr int kSkinnyMaxN = 16, kSkinnyMaxK = 1024, kSkinnyThreads = 256;

template <int NP>
__device__ __forceinline__ float lane_totals(float (&p)[NP], int lane) {
#pragma unroll
  for (int h = NP / 2; h >= 1; h /= 2) {
    bool up = lane & h;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      float send = up ? p[i] : p[i + h];
      p[i] = (up ? p[i + h] : p[i]) + __shfl_xor_sync(0xffffffffu, send, h);
    }
  }
  float v = p[0];
#pragma unroll
  for (int off = NP; off < 32; off <<= 1)
    v += __shfl_xor_sync(0xffffffffu, v, off);
  return v; // column lane & (NP - 1)
}

template <int NP, bool TransB>
__global__ void __launch_bounds__(kSkinnyThreads) skinny_kernel(int M, int N, int K, const float *__restrict__ A,
                                                              int lda, long long sA, const float *__restrict__ B,
                                                              int ldb, float *__restrict__ C, int ldc, long long sC) {
  extern __shared__ __align__(16) float bs[]; // [NP][KP], zero beyond N and K
  int KP = (K + 127) & ~127;
  A += blockIdx.y * sA;
  C += blockIdx.y * sC;
  for (int q = threadIdx.x; q < NP * KP; q += blockDim.x) {
    int nn = q / KP, k = q - nn * KP;
    bs[q] = nn < N && k < K ? (TransB ? B[size_t(nn) * ldb + k] : B[size_t(k) * ldb + nn]) : 0.f;
  }
  __syncthreads();
  int lane = threadIdx.x & 31;
  int warps = gridDim.x * (kSkinnyThreads / 32);
  for (int m = blockIdx.x * (kSkinnyThreads / 32) + (threadIdx.x >> 5); m < M; m += warps) {
    const float *a = A + size_t(m) * lda;
    float p[NP];
#pragma unroll
    for (int n = 0; n < NP; ++n)
      p[n] = 0.f;
    for (int k = 4 * lane; k < KP; k += 128) {
      float4 av = k < K ? *reinterpret_cast<const float4 *>(a + k) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int n = 0; n < NP; ++n) {
        float4 bv = *reinterpret_cast<const float4 *>(bs + n * KP + k);
        p[n] = fmaf(av.x, bv.x, fmaf(av.y, bv.y, fmaf(av.z, bv.z, fmaf(av.w, bv.w, p[n]))));
      }
    }
    float v = lane_totals<NP>(p, lane);
    if (lane < NP && lane < N)
      C[size_t(m) * ldc + lane] += v;
  }
}

// False when the shape or alignment does not suit skinny_kernel.
template <bool TransB>
bool launch_skinny(cudaStream_t s, int M, int N, int K, int batch, const float *A, int lda, long long sA,
                   const float *B, int ldb, float *C, int ldc, long long sC) {
  if (N > kSkinnyMaxN || K > kSkinnyMaxK || K % 4 || lda % 4 || sA % 4 || reinterpret_cast<uintptr_t>(A) % 16)
    return false;
  int np = N <= 1 ? 1 : N <= 2 ? 2 : N <= 4 ? 4 : N <= 8 ? 8 : 16;
  auto kernel = np == 1   ? skinny_kernel<1, TransB>
                : np == 2 ? skinny_kernel<2, TransB>
                : np == 4 ? skinny_kernel<4, TransB>
                : np == 8 ? skinny_kernel<8, TransB>
                          : skinny_kernel<16, TransB>;
  int smem = np * ((K + 127) & ~127) * 4;
  if (smem > 48 * 1024)
    lapis::check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  dim3 grid(std::min((M + kSkinnyThreads / 32 - 1) / (kSkinnyThreads / 32), 296), batch);
  lapis::launch(kernel, grid, kSkinnyThreads, smem, s, M, N, K, A, lda, sA, B, ldb, C, ldc, sC);
  return true;
}

__global__ void species_kernel(lapis::DeviceGeometry g, const int *lookup, int *species) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= g.n)
    return;
  int s = lookup[g.elements[i]];
  if (s < 0) {
    atomicCAS(g.status, 0, 2);
    s = 0;
  }
  species[i] = s;
}

__global__ void embed_kernel(int n, const int *species, const float *embedding, float *x) {
  size_t q = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (q >= size_t(n) * 512)
    return;
  int i = int(q / 512), c = int(q % 512);
  x[q] = embedding[species[i] * 512 + c];
}

// One thread per (node, 4 channels of 512): the 4 scalar groups and the 15 gated components,
// float4 accesses; every element follows the same FP32 expressions as a scalar pass.
__device__ __forceinline__ void ld4(const float *p, size_t k, float (&v)[4]) {
  float4 x = *reinterpret_cast<const float4 *>(p + k);
  v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w;
}
__device__ __forceinline__ void st4(float *p, size_t k, const float (&v)[4]) {
  *reinterpret_cast<float4 *>(p + k) = make_float4(v[0], v[1], v[2], v[3]);
}
// pre = raw / den + res for the 4 channels at k.
__device__ __forceinline__ void normalized4(const float *raw, const float *res, size_t k, float den, float (&u)[4]) {
  float r[4], q[4];
  ld4(raw, k, r);
  ld4(res, k, q);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    u[j] = r[j] / den + q[j];
}

// Four gate values at element k: fp32, or (gs set) as the tensor-core GEMM's split operand.
// The 16 lanes holding one 64-wide slab of a row (aligned groups of 16) reduce its maximum.
__device__ __forceinline__ void put4(float *gate, const SplitPlanes &gs, size_t k, const float (&v)[4], int lane) {
  if (!gs.hi) {
    st4(gate, k, v);
    return;
  }
  float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 1; o < 16; o <<= 1)
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  int e = tc::split_exponent(m);
  float2 sc = make_float2(__uint_as_float(uint32_t(127 + e) << 23), __uint_as_float(uint32_t(127 + e) << 23));
  float2 x0 = __fmul2_rn(make_float2(v[0], v[1]), sc), x1 = __fmul2_rn(make_float2(v[2], v[3]), sc);
  __half2 h0 = __float22half2_rn(x0), h1 = __float22half2_rn(x1);
  __half2 l0 = __float22half2_rn(__ffma2_rn(__half22float2(h0), make_float2(-1.f, -1.f), x0));
  __half2 l1 = __float22half2_rn(__ffma2_rn(__half22float2(h1), make_float2(-1.f, -1.f), x1));
  *reinterpret_cast<uint2 *>(gs.hi + k) =
      make_uint2(*reinterpret_cast<uint32_t *>(&h0), *reinterpret_cast<uint32_t *>(&h1));
  *reinterpret_cast<uint2 *>(gs.lo + k) =
      make_uint2(*reinterpret_cast<uint32_t *>(&l0), *reinterpret_cast<uint32_t *>(&l1));
  if (!(lane & 15))
    gs.exp[k / 64] = int16_t(e);
}

__global__ void normalize_gate_kernel(int n, const float *raw, const float *res, const float *rho, float alpha,
                                      float beta, float cs, float cg, float *gate, SplitPlanes gs) {
  int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= n * 128) // whole warps: 128 threads per node
    return;
  int i = q >> 7, c = (q & 127) * 4, lane = threadIdx.x & 31;
  float den = alpha + beta * rho[i];
  float u[4][4], o[4];
#pragma unroll
  for (int g = 0; g < 4; ++g)
    normalized4(raw, res, size_t(i) * 2048 + g * 512 + c, den, u[g]);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    o[j] = cs * u[0][j] * sigm(u[0][j]);
  put4(gate, gs, size_t(i) * 512 + c, o, lane);
#pragma unroll
  for (int l = 1; l <= 3; ++l) {
    float gl[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      gl[j] = sigm(u[l][j]);
#pragma unroll
    for (int m = l * l; m < (l + 1) * (l + 1); ++m) {
      float p[4];
      normalized4(raw, res, size_t(n) * 2048 + (size_t(m - 1) * n + i) * 512 + c, den, p);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o[j] = p[j] * cg * gl[j];
      put4(gate, gs, (size_t(m) * n + i) * 512 + c, o, lane);
    }
  }
}

// Four nodes per CTA, thread per 4 channels: gate VJP into pre_grad, normalisation VJP into
// raw_grad and density_grad (one fixed-order reduction per node).  pre is recomputed from raw
// and res; pg may alias res (each element is read before the same thread writes it).
__global__ void __launch_bounds__(512, 2) gate_norm_backward_kernel(int n, const float *res, const float *raw,
                                                                 const float *rho, const float *gg, float alpha,
                                                                 float beta, float cs, float cgt, float *pg,
                                                                 float *rg, float *rho_grad, SplitPlanes rgs) {
  __shared__ float red[4][4];
  int t = threadIdx.x, slot = t >> 7, c = (t & 127) * 4, i = blockIdx.x * 4 + slot, lane = t & 31;
  float s = 0.f;
  if (i < n) {
    float den = alpha + beta * rho[i];
    size_t k0 = size_t(i) * 2048 + c;
    float r[4], u[4], g[4], o[4], ro[4];
    ld4(raw, k0, r);
    normalized4(raw, res, k0, den, u);
    ld4(gg, size_t(i) * 512 + c, g);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float sg = sigm(u[j]);
      float g0 = g[j] * cs * sg * (1.f + u[j] * (1.f - sg));
      s -= g0 * r[j] * beta / (den * den);
      o[j] = g0;
      ro[j] = g0 / den;
    }
    st4(pg, k0, o);
    put4(rg, rgs, k0, ro, lane);
#pragma unroll
    for (int l = 1; l <= 3; ++l) {
      size_t gi = size_t(i) * 2048 + l * 512 + c;
      float gl[4], dg[4] = {0.f, 0.f, 0.f, 0.f}, rgi[4];
      normalized4(raw, res, gi, den, gl);
      ld4(raw, gi, rgi);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        gl[j] = sigm(gl[j]);
#pragma unroll
      for (int m = l * l; m < (l + 1) * (l + 1); ++m) {
        size_t src = size_t(n) * 2048 + (size_t(m - 1) * n + i) * 512 + c;
        float go[4], rs[4], qs[4];
        ld4(gg, (size_t(m) * n + i) * 512 + c, go);
        ld4(raw, src, rs);
        ld4(res, src, qs);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float v = go[j] * cgt * gl[j];
          dg[j] += go[j] * (rs[j] / den + qs[j]) * cgt * gl[j] * (1.f - gl[j]);
          s -= v * rs[j] * beta / (den * den);
          o[j] = v;
          ro[j] = v / den;
        }
        st4(pg, src, o);
        put4(rg, rgs, src, ro, lane);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s -= dg[j] * rgi[j] * beta / (den * den);
        o[j] = dg[j];
        ro[j] = dg[j] / den;
      }
      st4(pg, gi, o);
      put4(rg, rgs, gi, ro, lane);
    }
  }
#pragma unroll
  for (int step = 16; step; step >>= 1)
    s += __shfl_xor_sync(0xffffffffu, s, step);
  if ((t & 31) == 0)
    red[slot][(t >> 5) & 3] = s;
  __syncthreads();
  if ((t & 127) == 0 && i < n)
    rho_grad[i] = (red[slot][0] + red[slot][1]) + (red[slot][2] + red[slot][3]);
}

// Symmetric contraction: y[out][c] = sum_t coef[t][c] x[a][c] x[b][c] x[c'][c] (degree <= 3).
// CTA = 8 warps owning a 32-channel slice: the slice of every coefficient row and the term
// table are staged in shared memory once, then each warp streams nodes (lane = channel) with
// the node's 16 components plus a constant 1 (index 16) in a per-warp shared array.  Terms
// are sorted by output at load and their missing factors point at the constant, so every
// term is the same branch-free coef * v[a] * v[b] * v[c]; four independent partial sums keep
// the dependent shared-memory loads overlapped.
constexpr int kProdWarps = 8, kProdNodes = 64, kProdV = 17;

__global__ void __launch_bounds__(256) product_kernel(int n, const int *abc, const float *coef, int count,
                                                      const int4 out_start, int outputs, const float *x, float *y) {
  extern __shared__ float ps[];
  float *cs = ps;                                     // [count][32]
  int *ts = reinterpret_cast<int *>(cs + count * 32); // [count]  a | b << 8 | c << 16
  float *vs = reinterpret_cast<float *>(ts + ((count + 3) & ~3)) + (threadIdx.x >> 5) * kProdV * 32;
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, c0 = blockIdx.x * 32;
  for (int k = threadIdx.x; k < count * 32; k += blockDim.x)
    cs[k] = coef[size_t(k >> 5) * 512 + c0 + (k & 31)];
  for (int k = threadIdx.x; k < count; k += blockDim.x)
    ts[k] = abc[k];
  vs[16 * 32 + lane] = 1.f;
  __syncthreads();
  int bounds[5] = {out_start.x, out_start.y, out_start.z, out_start.w, count};
  int i0 = blockIdx.y * kProdNodes, i1 = min(n, i0 + kProdNodes);
  for (int i = i0 + warp; i < i1; i += kProdWarps) {
#pragma unroll
    for (int m = 0; m < 16; ++m)
      vs[m * 32 + lane] = x[(size_t(m) * n + i) * 512 + c0 + lane];
    __syncwarp();
    for (int o = 0; o < outputs; ++o) {
      int k = bounds[o], end = bounds[o + 1];
      float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
      for (; k + 4 <= end; k += 4) {
        int t0 = ts[k], t1 = ts[k + 1], t2 = ts[k + 2], t3 = ts[k + 3];
        s0 = fmaf(cs[k * 32 + lane] * vs[(t0 & 255) * 32 + lane],
                  vs[((t0 >> 8) & 255) * 32 + lane] * vs[(t0 >> 16) * 32 + lane], s0);
        s1 = fmaf(cs[(k + 1) * 32 + lane] * vs[(t1 & 255) * 32 + lane],
                  vs[((t1 >> 8) & 255) * 32 + lane] * vs[(t1 >> 16) * 32 + lane], s1);
        s2 = fmaf(cs[(k + 2) * 32 + lane] * vs[(t2 & 255) * 32 + lane],
                  vs[((t2 >> 8) & 255) * 32 + lane] * vs[(t2 >> 16) * 32 + lane], s2);
        s3 = fmaf(cs[(k + 3) * 32 + lane] * vs[(t3 & 255) * 32 + lane],
                  vs[((t3 >> 8) & 255) * 32 + lane] * vs[(t3 >> 16) * 32 + lane], s3);
      }
      for (; k < end; ++k) {
        int t0 = ts[k];
        s0 = fmaf(cs[k * 32 + lane] * vs[(t0 & 255) * 32 + lane],
                  vs[((t0 >> 8) & 255) * 32 + lane] * vs[(t0 >> 16) * 32 + lane], s0);
      }
      y[(size_t(o) * n + i) * 512 + c0 + lane] = (s0 + s1) + (s2 + s3);
    }
    __syncwarp();
  }
}

// VJP: g[a] += w G b c, g[b] += w G a c, g[c] += w G a b (missing factors are the constant 1,
// whose gradient slot 16 is a discard).
__global__ void __launch_bounds__(256) product_backward_kernel(int n, const int *abc, const float *coef, int count,
                                                               const int4 out_start, int outputs, const float *x,
                                                               const float *grad, float *xg) {
  extern __shared__ float ps[];
  float *cs = ps;
  int *ts = reinterpret_cast<int *>(cs + count * 32);
  float *vs = reinterpret_cast<float *>(ts + ((count + 3) & ~3)) + (threadIdx.x >> 5) * 2 * kProdV * 32;
  float *gs = vs + kProdV * 32;
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, c0 = blockIdx.x * 32;
  for (int k = threadIdx.x; k < count * 32; k += blockDim.x)
    cs[k] = coef[size_t(k >> 5) * 512 + c0 + (k & 31)];
  for (int k = threadIdx.x; k < count; k += blockDim.x)
    ts[k] = abc[k];
  vs[16 * 32 + lane] = 1.f;
  __syncthreads();
  int bounds[5] = {out_start.x, out_start.y, out_start.z, out_start.w, count};
  int i0 = blockIdx.y * kProdNodes, i1 = min(n, i0 + kProdNodes);
  for (int i = i0 + warp; i < i1; i += kProdWarps) {
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      vs[m * 32 + lane] = x[(size_t(m) * n + i) * 512 + c0 + lane];
      gs[m * 32 + lane] = 0.f;
    }
    __syncwarp();
    for (int o = 0; o < outputs; ++o) {
      float G = grad[(size_t(o) * n + i) * 512 + c0 + lane];
      for (int k = bounds[o]; k < bounds[o + 1]; ++k) {
        int t = ts[k], ia = (t & 255) * 32 + lane, ib = ((t >> 8) & 255) * 32 + lane, ic = (t >> 16) * 32 + lane;
        float gw = cs[k * 32 + lane] * G;
        float a = vs[ia], b = vs[ib], d = vs[ic];
        gs[ia] += gw * b * d;
        gs[ib] += gw * a * d;
        gs[ic] += gw * a * b;
      }
    }
    __syncwarp();
#pragma unroll
    for (int m = 0; m < 16; ++m)
      xg[(size_t(m) * n + i) * 512 + c0 + lane] = gs[m * 32 + lane];
    __syncwarp();
  }
}

// Compiled product basis (product_table.h): the term structure is known at compile time,
// so a thread keeps its nodes' 16 components (plus the constant 1 at index 16) and their
// gradients in registers and every term is ((coef * v[a]) * v[b]) * v[c] with constant
// indices.  Every partial product carries the term's own coefficient, so no product is
// shared between terms and only the components and gradients stay live.  Thread = channel
// of a 32-channel slice, two nodes at a time so each coefficient read from shared memory
// serves both.
template <int L> struct PolyTable;
template <> struct PolyTable<0> {
  static constexpr int NT = kPolyTerms0, NOUT = 4;
  static constexpr int start(int o) { return kPolyStart0[o]; }
  static constexpr PolyABC term(int k) { return kPoly0[k]; }
};
template <> struct PolyTable<1> {
  static constexpr int NT = kPolyTerms1, NOUT = 1;
  static constexpr int start(int o) { return kPolyStart1[o]; }
  static constexpr PolyABC term(int k) { return kPoly1[k]; }
};
template <int I, int N> struct PUnroll {
  template <class F> __device__ __forceinline__ static void run(F &&f) {
    f(std::integral_constant<int, I>{});
    PUnroll<I + 1, N>::run(f);
  }
};
template <int N> struct PUnroll<N, N> {
  template <class F> __device__ __forceinline__ static void run(F &&) {}
};
constexpr int kPolyPair = 2; // nodes per thread
constexpr int kPolyWarps = 4;

// Nested evaluation over the (a, b, c)-sorted terms of one output:
//     y = sum_a v_a T_a,   T_a = sum_b v_b S_ab,   S_ab = sum_c cf_abc v_c
// -- one FP32 operation per term plus one per (a, b) group and per a group -- and its VJP
// with the output gradient G:
//     g_c += cf_abc (G v_a v_b),   g_b += (G v_a) S_ab,   g_a += G T_a.
// Missing factors are the constant slot 16 (v = 1; its gradient is discarded).
template <int L> constexpr bool poly_same_a(int s, int t) { return PolyTable<L>::term(s).a == PolyTable<L>::term(t).a; }
template <int L> constexpr bool poly_same_ab(int s, int t) {
  return poly_same_a<L>(s, t) && PolyTable<L>::term(s).b == PolyTable<L>::term(t).b;
}
// First term of the a group / (a, b) group that term k of output o belongs to.
template <int L> constexpr int a_head(int o, int k) {
  while (k > PolyTable<L>::start(o) && poly_same_a<L>(k - 1, k))
    --k;
  return k;
}
template <int L> constexpr int ab_head(int o, int k) {
  while (k > PolyTable<L>::start(o) && poly_same_ab<L>(k - 1, k))
    --k;
  return k;
}
template <int L> constexpr bool a_end(int o, int k) {
  return k + 1 == PolyTable<L>::start(o + 1) || !poly_same_a<L>(k, k + 1);
}
template <int L> constexpr bool ab_end(int o, int k) {
  return k + 1 == PolyTable<L>::start(o + 1) || !poly_same_ab<L>(k, k + 1);
}
template <int L> constexpr bool poly_groups_contiguous() {
  using PT = PolyTable<L>;
  for (int o = 0; o < PT::NOUT; ++o)
    for (int s = PT::start(o); s < PT::start(o + 1); ++s)
      for (int t = s + 1; t < PT::start(o + 1); ++t)
        if ((poly_same_a<L>(s, t) && !poly_same_a<L>(t - 1, t)) ||
            (poly_same_ab<L>(s, t) && !poly_same_ab<L>(t - 1, t)))
          return false;
  return true;
}
static_assert(poly_groups_contiguous<0>() && poly_groups_contiguous<1>(), "product terms must be (a, b, c)-sorted");

// Split (backward only): the input gradient goes out as SplitPlanes.  A CTA then covers 64
// channels -- one 64-wide slab of each row -- as two halves of 32, each taken by half of the
// warps; the two warps of a node pair exchange their 32-channel maxima through shared memory.
template <int L, bool Bwd, bool Split = false>
__global__ void __launch_bounds__(32 * kPolyWarps, Bwd || L == 0 ? 2 : 3)
    product_fixed_kernel(int n, const float *coef, const float *x, const float *grad, float *y, SplitPlanes ys) {
  // The thread's two nodes travel as float2 pairs, so every FMA and product below is one paired
  // instruction (fma.rn.f32x2 / mul.rn.f32x2: two IEEE operations).
  static_assert(kPolyPair == 2, "paired evaluation assumes two nodes per thread");
  static_assert(!Split || Bwd, "only the backward writes a split output");
  using PT = PolyTable<L>;
  constexpr int kCh = Split ? 64 : 32, kSlots = Split ? kPolyWarps / 2 : kPolyWarps; // channels; warps per half
  extern __shared__ float cs[]; // [NT][kCh]
  __shared__ float xch[Split ? 2 : 1][kSlots][2][16][2]; // [buffer][slot][half][component][node]: maxima
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, half = warp / kSlots, slot = warp % kSlots;
  int cb = blockIdx.x * kCh, c0 = cb + 32 * half; // the CTA's first channel; this warp's
  for (int k = threadIdx.x; k < PT::NT * kCh; k += blockDim.x)
    cs[k] = coef[size_t(k / kCh) * 512 + cb + (k % kCh)];
  __syncthreads();
  int i0 = blockIdx.y * kProdNodes, i1 = min(n, i0 + kProdNodes), it = 0;
  for (int ib = i0 + slot * kPolyPair; ib < i1; ib += kSlots * kPolyPair, ++it) {
    bool second = ib + 1 < i1;
    float2 v[17];
#pragma unroll
    for (int m = 0; m < 16; ++m)
      v[m] = make_float2(x[(size_t(m) * n + ib) * 512 + c0 + lane],
                         second ? x[(size_t(m) * n + ib + 1) * 512 + c0 + lane] : 0.f);
    v[16] = make_float2(1.f, 1.f);
    if constexpr (!Bwd) {
      PUnroll<0, PT::NOUT>::run([&](auto oc) {
        constexpr int o = decltype(oc)::value;
        float2 acc, T, S;
        PUnroll<PT::start(o), PT::start(o + 1)>::run([&](auto kc) {
          constexpr int k = decltype(kc)::value;
          constexpr PolyABC t = PT::term(k);
          constexpr int ab0 = ab_head<L>(o, k), a0 = a_head<L>(o, k);
          float cf = cs[k * kCh + 32 * half + lane];
          float2 cf2 = make_float2(cf, cf);
          S = k == ab0 ? __fmul2_rn(cf2, v[t.c]) : __ffma2_rn(cf2, v[t.c], S);
          if constexpr (ab_end<L>(o, k))
            T = ab0 == a0 ? __fmul2_rn(v[t.b], S) : __ffma2_rn(v[t.b], S, T);
          if constexpr (a_end<L>(o, k))
            acc = a0 == PT::start(o) ? __fmul2_rn(v[t.a], T) : __ffma2_rn(v[t.a], T, acc);
        });
        y[(size_t(o) * n + ib) * 512 + c0 + lane] = acc.x;
        if (second)
          y[(size_t(o) * n + ib + 1) * 512 + c0 + lane] = acc.y;
      });
    } else {
      float2 g[17];
#pragma unroll
      for (int m = 0; m < 17; ++m)
        g[m] = make_float2(0.f, 0.f);
      PUnroll<0, PT::NOUT>::run([&](auto oc) {
        constexpr int o = decltype(oc)::value;
        float2 G = make_float2(grad[(size_t(o) * n + ib) * 512 + c0 + lane],
                               second ? grad[(size_t(o) * n + ib + 1) * 512 + c0 + lane] : 0.f);
        float2 Gva, u, T, S;
        PUnroll<PT::start(o), PT::start(o + 1)>::run([&](auto kc) {
          constexpr int k = decltype(kc)::value;
          constexpr PolyABC t = PT::term(k);
          constexpr int ab0 = ab_head<L>(o, k), a0 = a_head<L>(o, k);
          float cf = cs[k * kCh + 32 * half + lane];
          float2 cf2 = make_float2(cf, cf);
          if constexpr (k == a0)
            Gva = __fmul2_rn(G, v[t.a]);
          if constexpr (k == ab0)
            u = __fmul2_rn(Gva, v[t.b]);
          S = k == ab0 ? __fmul2_rn(cf2, v[t.c]) : __ffma2_rn(cf2, v[t.c], S);
          g[t.c] = __ffma2_rn(cf2, u, g[t.c]);
          if constexpr (ab_end<L>(o, k)) {
            g[t.b] = __ffma2_rn(Gva, S, g[t.b]);
            T = ab0 == a0 ? __fmul2_rn(v[t.b], S) : __ffma2_rn(v[t.b], S, T);
          }
          if constexpr (a_end<L>(o, k))
            g[t.a] = __ffma2_rn(G, T, g[t.a]);
        });
      });
      if constexpr (Split) {
        float(*mx)[2][16][2] = xch[it & 1]; // [slot][half][component][node]
        // Warp maxima of |g| as integer reductions of the bit patterns (ordered like the values
        // for non-negative floats).
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          unsigned a = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(g[m].x)));
          unsigned b = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(g[m].y)));
          if (lane == 0)
            mx[slot][half][m][0] = __uint_as_float(a), mx[slot][half][m][1] = __uint_as_float(b);
        }
        // The two warps of this node pair (one per half) meet here, once per iteration; the
        // maxima are double-buffered, so the next iteration's writes cannot race these reads.
        static_assert(kSlots == 2, "one named barrier per node-pair slot");
        if (slot == 0)
          asm volatile("bar.sync 1, 64;" ::: "memory");
        else
          asm volatile("bar.sync 2, 64;" ::: "memory");
#pragma unroll
        for (int m = 0; m < 16; ++m)
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            if (q && !second)
              continue;
            int e = tc::split_exponent(fmaxf(mx[slot][0][m][q], mx[slot][1][m][q]));
            float x2 = (q ? g[m].y : g[m].x) * __uint_as_float(uint32_t(127 + e) << 23);
            __half h = __float2half_rn(x2), l = __float2half_rn(x2 - __half2float(h));
            size_t el = (size_t(m) * n + ib + q) * 512 + c0 + lane;
            ys.hi[el] = __half_as_ushort(h);
            ys.lo[el] = __half_as_ushort(l);
            if (half == 0 && lane == 0)
              ys.exp[el / 64] = int16_t(e);
          }
      } else {
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          y[(size_t(m) * n + ib) * 512 + c0 + lane] = g[m].x;
          if (second)
            y[(size_t(m) * n + ib + 1) * 512 + c0 + lane] = g[m].y;
        }
      }
    }
  }
}

__global__ void add_kernel(size_t count, const float *a, float *b, float scale) {
  size_t k = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (k < count)
    b[k] += scale * a[k];
}
__global__ void fill_kernel(size_t count, float *a, float value) {
  size_t k = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (k < count)
    a[k] = value;
}
__global__ void readout_act_kernel(int count, const float *x, const float *grad, float *y, float scale,
                                   bool backward) {
  int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= count)
    return;
  float s = sigm(x[k]);
  y[k] = backward ? grad[k] * scale * s * (1.f + x[k] * (1.f - s)) : scale * x[k] * s;
}

unsigned blocks_for(size_t count, int threads) { return unsigned((count + threads - 1) / threads); }
} // namespace

void launch_species(cudaStream_t s, const lapis::DeviceGeometry &g, const int *lookup, int *species) {
  if (g.n)
    lapis::launch(species_kernel, blocks_for(g.n, 256), 256, 0, s, g, lookup, species);
}
void launch_embed(cudaStream_t s, int n, const int *species, const float *embedding, float *x) {
  if (n)
    lapis::launch(embed_kernel, blocks_for(size_t(n) * 512, 256), 256, 0, s, n, species, embedding, x);
}

bool tensor_core_linears() {
  static const bool on = [] {
    const char *v = std::getenv("MACE_SIMT_LINEARS");
    return !(v && v[0] == '1');
  }();
  return on;
}

bool projection_edges() {
  static const bool on = [] {
    const char *v = std::getenv("MACE_SIMT_EDGES");
    return tensor_core_linears() && !(v && v[0] == '1');
  }();
  return on;
}

bool linear_takes_split(const Linear &l, bool backward) {
  if (!tensor_core_linears())
    return false;
  for (size_t q = 0; q < l.paths.size(); ++q)
    if (!(backward ? l.tc[q].bwd : l.tc[q].fwd) || (backward ? l.paths[q].out_mul : l.paths[q].in_mul) % 64)
      return false;
  return !l.paths.empty();
}

void linear(cudaStream_t s, int n, const Linear &l, const float *x, float *y, bool backward, bool add, int *status,
            int nx, int ny, const SplitPlanes *xs) {
  if (!n)
    return;
  if (!nx)
    nx = n;
  if (!ny)
    ny = n;
  bool tc = tensor_core_linears() && status;
  if (xs && (!tc || !linear_takes_split(l, backward)))
    throw lapis::Error("linear: a split input needs every path on the tensor cores");
  // Tensor-core paths: paths writing the same output block become one GEMM whose K range
  // concatenates their inputs (segments in path order); the resulting problems go out as
  // grouped launches.  When every path runs on the tensor cores and the blocks tile the
  // output, the GEMMs store directly (no zero fill, no read-modify-write).
  struct Problem {
    int o0, o1;
    std::vector<GemmSpec> segs;
  };
  std::vector<Problem> problems;
  bool all_tc = tc, overlap = false;
  for (size_t q = 0; q < l.paths.size(); ++q) {
    const auto &p = l.paths[q];
    const TCWeights &t = l.tc[q];
    if (!tc || !(backward ? t.bwd : t.fwd)) {
      all_tc = false;
      continue;
    }
    int o0 = backward ? p.in_offset : p.out_offset, o1 = o0 + (backward ? p.in_mul : p.out_mul) * p.dim;
    GemmSpec g = !backward ? GemmSpec{n, p.out_mul, p.in_mul, p.dim, x + size_t(p.in_offset) * nx,
                                      (long long)nx * p.in_mul, t.fwd, y + size_t(p.out_offset) * ny,
                                      p.out_mul, (long long)ny * p.out_mul, true}
                           : GemmSpec{n, p.in_mul, p.out_mul, p.dim, x + size_t(p.out_offset) * nx,
                                      (long long)nx * p.out_mul, t.bwd, y + size_t(p.in_offset) * ny,
                                      p.in_mul, (long long)ny * p.in_mul, true};
    if (xs) { // the same elements in the split planes; one exponent per 64 of them
      size_t off = size_t(backward ? p.out_offset : p.in_offset) * nx;
      g.Ahi = xs->hi + off;
      g.Alo = xs->lo + off;
      g.Aexp = xs->exp + off / 64;
      g.strideAexp = g.strideA / 64;
    }
    Problem *same = nullptr;
    for (auto &pr : problems) {
      if (pr.o0 == o0 && pr.o1 == o1 && pr.segs[0].N == g.N && pr.segs[0].batch == g.batch)
        same = &pr;
      else if (o0 < pr.o1 && pr.o0 < o1)
        overlap = true;
    }
    if (same)
      same->segs.push_back(g);
    else
      problems.push_back(Problem{o0, o1, {g}});
  }
  long long covered = 0;
  for (auto &pr : problems)
    covered += pr.o1 - pr.o0;
  bool store = !add && all_tc && !overlap && covered == (backward ? l.input : l.output);
  if (!add && !store)
    lapis::check(cudaMemsetAsync(y, 0, size_t(ny) * (backward ? l.input : l.output) * 4, s));
  // Problems whose blocks partly overlap stay in separate launches, in path order.
  std::vector<GemmSpec> group;
  std::vector<std::pair<int, int>> ranges;
  for (auto &pr : problems) {
    for (auto &r : ranges)
      if (pr.o0 < r.second && r.first < pr.o1) {
        tc_gemm_group(s, group.data(), int(group.size()), status);
        group.clear();
        ranges.clear();
        break;
      }
    ranges.push_back({pr.o0, pr.o1});
    for (size_t k = 0; k < pr.segs.size(); ++k) {
      GemmSpec g = pr.segs[k];
      g.accumulate = !store;
      g.join = k > 0;
      group.push_back(g);
    }
  }
  if (!group.empty())
    tc_gemm_group(s, group.data(), int(group.size()), status);
  // The remaining paths on the FP32 SIMT kernels (accumulating).
  for (size_t q = 0; q < l.paths.size(); ++q) {
    const auto &p = l.paths[q];
    const float *w = l.weight + p.weight_offset;
    const TCWeights &t = l.tc[q];
    if (tc && (backward ? t.bwd : t.fwd))
      continue;
    if (!backward) {
      if (launch_skinny<false>(s, n, p.out_mul, p.in_mul, p.dim, x + size_t(p.in_offset) * nx, p.in_mul,
                               (long long)nx * p.in_mul, w, p.out_mul, y + size_t(p.out_offset) * ny, p.out_mul,
                               (long long)ny * p.out_mul))
        continue;
      dim3 grid((p.out_mul + BN - 1) / BN, (n + BM - 1) / BM, p.dim);
      lapis::launch(gemm_kernel<false>, grid, 256, 0, s, n, p.out_mul, p.in_mul, x + size_t(p.in_offset) * nx,
                    p.in_mul, (long long)nx * p.in_mul, w, p.out_mul, y + size_t(p.out_offset) * ny, p.out_mul,
                    (long long)ny * p.out_mul);
    } else {
      if (launch_skinny<true>(s, n, p.in_mul, p.out_mul, p.dim, x + size_t(p.out_offset) * nx, p.out_mul,
                              (long long)nx * p.out_mul, w, p.out_mul, y + size_t(p.in_offset) * ny, p.in_mul,
                              (long long)ny * p.in_mul))
        continue;
      dim3 grid((p.in_mul + BN - 1) / BN, (n + BM - 1) / BM, p.dim);
      lapis::launch(gemm_kernel<true>, grid, 256, 0, s, n, p.in_mul, p.out_mul, x + size_t(p.out_offset) * nx,
                    p.out_mul, (long long)nx * p.out_mul, w, p.out_mul, y + size_t(p.in_offset) * ny, p.in_mul,
                    (long long)ny * p.in_mul);
    }
  }
}

void launch_normalize_gate(cudaStream_t s, int n, const float *raw, const float *res, const float *density,
                           float alpha, float beta, float scalar_scale, float gate_scale, float *gate,
                           SplitPlanes gs) {
  if (n)
    lapis::launch(normalize_gate_kernel, blocks_for(size_t(n) * 128, 256), 256, 0, s, n, raw, res, density, alpha, beta,
                  scalar_scale, gate_scale, gate, gs);
}
void launch_gate_norm_backward(cudaStream_t s, int n, const float *res, const float *raw, const float *density,
                               const float *gate_grad, float alpha, float beta, float scalar_scale, float gate_scale,
                               float *pre_grad, float *raw_grad, float *density_grad, SplitPlanes raw_grad_split) {
  if (n)
    lapis::launch(gate_norm_backward_kernel, (n + 3) / 4, 512, 0, s, n, res, raw, density, gate_grad, alpha, beta,
                  scalar_scale, gate_scale, pre_grad, raw_grad, density_grad, raw_grad_split);
}
size_t product_smem(int count, bool backward) {
  return (size_t(count) * 32 + ((count + 3) & ~3)) * 4 + size_t(kProdWarps) * (backward ? 2 : 1) * kProdV * 32 * 4;
}

template <int L, bool Bwd, bool Split = false>
void launch_product_fixed(cudaStream_t s, int n, const Layer &l, const float *x, const float *grad, float *y,
                          SplitPlanes ys = {}) {
  constexpr int kCh = Split ? 64 : 32;
  int smem = PolyTable<L>::NT * kCh * 4;
  auto kernel = product_fixed_kernel<L, Bwd, Split>;
  lapis::check(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  dim3 grid(512 / kCh, (n + kProdNodes - 1) / kProdNodes);
  lapis::launch(kernel, grid, 32 * kPolyWarps, smem, s, n, l.poly_coef_sorted, x, grad, y, ys);
}

void launch_product(cudaStream_t s, int n, const Layer &l, const float *x, float *y) {
  if (!n)
    return;
  if (l.poly_fixed >= 0) {
    if (l.poly_fixed == 0)
      launch_product_fixed<0, false>(s, n, l, x, nullptr, y);
    else
      launch_product_fixed<1, false>(s, n, l, x, nullptr, y);
    return;
  }
  size_t smem = product_smem(l.npoly, false);
  lapis::check(cudaFuncSetAttribute(product_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  dim3 grid(16, (n + kProdNodes - 1) / kProdNodes);
  lapis::launch(product_kernel, grid, 256, smem, s, n, l.poly_abc, l.poly_coef_sorted, l.npoly, l.poly_out_start,
                l.pouts, x, y);
}
void launch_product_backward(cudaStream_t s, int n, const Layer &l, const float *x, const float *grad, float *xg,
                             SplitPlanes xgs) {
  if (!n)
    return;
  if (xgs.hi && l.poly_fixed < 0)
    throw lapis::Error("a split product gradient needs the compiled product tables");
  if (l.poly_fixed >= 0) {
    if (xgs.hi) {
      if (l.poly_fixed == 0)
        launch_product_fixed<0, true, true>(s, n, l, x, grad, xg, xgs);
      else
        launch_product_fixed<1, true, true>(s, n, l, x, grad, xg, xgs);
    } else if (l.poly_fixed == 0) {
      launch_product_fixed<0, true>(s, n, l, x, grad, xg);
    } else {
      launch_product_fixed<1, true>(s, n, l, x, grad, xg);
    }
    return;
  }
  size_t smem = product_smem(l.npoly, true);
  lapis::check(
      cudaFuncSetAttribute(product_backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  dim3 grid(16, (n + kProdNodes - 1) / kProdNodes);
  lapis::launch(product_backward_kernel, grid, 256, smem, s, n, l.poly_abc, l.poly_coef_sorted, l.npoly,
                l.poly_out_start, l.pouts, x, grad, xg);
}
void launch_add(cudaStream_t s, size_t count, const float *a, float *b, float scale) {
  if (count)
    lapis::launch(add_kernel, blocks_for(count, 256), 256, 0, s, count, a, b, scale);
}
void launch_fill(cudaStream_t s, size_t count, float *a, float value) {
  if (count)
    lapis::launch(fill_kernel, blocks_for(count, 256), 256, 0, s, count, a, value);
}
void launch_readout_act(cudaStream_t s, int count, const float *x, const float *grad, float *y, float scale,
                        bool backward) {
  if (count)
    lapis::launch(readout_act_kernel, blocks_for(count, 256), 256, 0, s, count, x, grad, y, scale, backward);
}
} // namespace mace

namespace lapis {
void set_c_api_error(const std::string &message);
}

extern "C" int mace_debug_gemm(int M, int N, int K, int batch, const float *A, const float *B, float *C,
                               int accumulate, int mode) {
  using namespace mace;
  std::vector<void *> owned; // device buffers of this call
  int *status = nullptr;
  auto alloc = [&](size_t bytes) {
    void *p = nullptr;
    lapis::check(cudaMalloc(&p, bytes));
    owned.push_back(p);
    return p;
  };
  auto release = [&] {
    for (void *p : owned)
      cudaFree(p);
    owned.clear();
  };
  // The fp16 split of a K-major [n][k] host matrix, on the device.
  auto split = [&](const float *bt, int n, int k) {
    std::vector<uint16_t> h(size_t(n) * k), l(h.size());
    TCMatrix m;
    m.exp = split_f16(bt, h.size(), h.data(), l.data());
    auto *hd = static_cast<uint16_t *>(alloc(h.size() * 2)), *ld = static_cast<uint16_t *>(alloc(l.size() * 2));
    lapis::check(cudaMemcpy(hd, h.data(), h.size() * 2, cudaMemcpyHostToDevice));
    lapis::check(cudaMemcpy(ld, l.data(), l.size() * 2, cudaMemcpyHostToDevice));
    m.hi = hd;
    m.lo = ld;
    return m;
  };
  try {
    lapis::set_c_api_error("");
    if (M < 0 || N <= 0 || K <= 0 || batch <= 0 || !A || !B || !C)
      throw lapis::Error("Invalid GEMM arguments");
    if (mode == 0) {
      if (!accumulate)
        lapis::check(cudaMemset(C, 0, size_t(batch) * M * N * 4));
      dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM, batch);
      lapis::launch(gemm_kernel<false>, grid, 256, 0, cudaStream_t(0), M, N, K, A, K, (long long)M * K, B, N, C, N,
                    (long long)M * N);
    } else {
      std::vector<float> b(size_t(K) * N), bt(b.size());
      lapis::check(cudaMemcpy(b.data(), B, b.size() * 4, cudaMemcpyDeviceToHost));
      for (int k = 0; k < K; ++k)
        for (int n = 0; n < N; ++n)
          bt[size_t(n) * K + k] = b[size_t(k) * N + n];
      status = static_cast<int *>(alloc(4));
      lapis::check(cudaMemset(status, 0, 4));
      if (mode == 1) {
        TCMatrix m = split(bt.data(), N, K);
        tc_gemm(cudaStream_t(0), M, N, K, batch, A, (long long)M * K, m, C, N, (long long)M * N, accumulate != 0,
                status);
      } else if (mode == 4) { // A given as split planes, made here by the host rule
        if (K % 64)
          throw lapis::Error("mode 4 needs K a multiple of 64");
        std::vector<float> ah(size_t(batch) * M * K);
        lapis::check(cudaMemcpy(ah.data(), A, ah.size() * 4, cudaMemcpyDeviceToHost));
        std::vector<uint16_t> hi(ah.size()), lo(ah.size());
        std::vector<int16_t> ex(ah.size() / 64);
        for (size_t b = 0; b < ex.size(); ++b) {
          float mx = 0.f;
          for (int k = 0; k < 64; ++k)
            mx = std::max(mx, std::fabs(ah[b * 64 + k]));
          int e = 0;
          if (mx > 0.f) {
            int x2 = 0;
            std::frexp(mx, &x2);
            e = std::min(100, std::max(-100, 15 - x2));
          }
          ex[b] = int16_t(e);
          for (int k = 0; k < 64; ++k) {
            float x = std::ldexp(ah[b * 64 + k], e);
            __half h = __float2half_rn(x), l = __float2half_rn(x - __half2float(h));
            std::memcpy(&hi[b * 64 + k], &h, 2);
            std::memcpy(&lo[b * 64 + k], &l, 2);
          }
        }
        auto *hd = static_cast<uint16_t *>(alloc(hi.size() * 2)), *ld = static_cast<uint16_t *>(alloc(lo.size() * 2));
        auto *xd = static_cast<int16_t *>(alloc(ex.size() * 2));
        lapis::check(cudaMemcpy(hd, hi.data(), hi.size() * 2, cudaMemcpyHostToDevice));
        lapis::check(cudaMemcpy(ld, lo.data(), lo.size() * 2, cudaMemcpyHostToDevice));
        lapis::check(cudaMemcpy(xd, ex.data(), ex.size() * 2, cudaMemcpyHostToDevice));
        GemmSpec g{M, N, K, batch, A, (long long)M * K, split(bt.data(), N, K), C, N, (long long)M * N,
                   accumulate != 0};
        g.Ahi = hd, g.Alo = ld, g.Aexp = xd, g.strideAexp = (long long)M * K / 64;
        tc_gemm_group(cudaStream_t(0), &g, 1, status);
      } else if (mode == 3) { // K split into two segments with their own contiguous A and B
        int k0 = (K / 64) * 32, k1 = K - k0;
        if (!k0)
          throw lapis::Error("mode 3 needs K >= 64");
        std::vector<float> ah(size_t(batch) * M * K);
        lapis::check(cudaMemcpy(ah.data(), A, ah.size() * 4, cudaMemcpyDeviceToHost));
        GemmSpec g[2];
        for (int q = 0; q < 2; ++q) {
          int kb = q ? k0 : 0, kc = q ? k1 : k0;
          // Segment q's B is scaled by 2^(8 q) and its A by 2^-(8 q) (products unchanged), so
          // that the segments carry different B exponents.
          std::vector<float> bs(size_t(N) * kc), as(size_t(batch) * M * kc);
          for (int n = 0; n < N; ++n)
            for (int k = 0; k < kc; ++k)
              bs[size_t(n) * kc + k] = std::ldexp(bt[size_t(n) * K + kb + k], 8 * q);
          for (size_t r = 0; r < size_t(batch) * M; ++r)
            for (int k = 0; k < kc; ++k)
              as[r * kc + k] = std::ldexp(ah[r * K + kb + k], -8 * q);
          auto *a = static_cast<float *>(alloc(as.size() * 4 + 16));
          lapis::check(cudaMemcpy(a, as.data(), as.size() * 4, cudaMemcpyHostToDevice));
          g[q] = GemmSpec{M, N, kc, batch, a, (long long)M * kc, split(bs.data(), N, kc), C, N, (long long)M * N,
                          accumulate != 0, q == 1};
        }
        tc_gemm_group(cudaStream_t(0), g, 2, status);
      } else { // grouped: one problem per batch plane, columns split as [128, N - 128]
        TCMatrix m = split(bt.data(), N, K);
        std::vector<GemmSpec> group;
        for (int z = 0; z < batch; ++z)
          for (int n0 = 0; n0 < N; n0 += (n0 ? N : 128)) {
            int nc = n0 ? N - n0 : std::min(N, 128);
            TCMatrix part{m.hi + size_t(n0) * K, m.lo + size_t(n0) * K, m.exp};
            group.push_back(GemmSpec{M, nc, K, 1, A + size_t(z) * M * K, (long long)M * K, part,
                                     C + size_t(z) * M * N + n0, N, (long long)M * N, accumulate != 0});
          }
        tc_gemm_group(cudaStream_t(0), group.data(), int(group.size()), status);
      }
    }
    lapis::check(cudaGetLastError());
    lapis::check(cudaDeviceSynchronize());
    int st = 0;
    if (status)
      lapis::check(cudaMemcpy(&st, status, 4, cudaMemcpyDeviceToHost));
    release();
    if (st)
      throw lapis::Error("tensor-core GEMM reported status " + std::to_string(st));
    return 0;
  } catch (const std::exception &e) {
    cudaDeviceSynchronize();
    release();
    lapis::set_c_api_error(e.what());
    return -1;
  }
}
