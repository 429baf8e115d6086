// MH1 edge kernels for B200 (FP32, CSR edges from the Lapis runtime).
//
// Mathematics follows the reference (LipidL/LASP-PIS mace/src/mh1.cu, mh1_math.cuh):
//   Agnesi transform + Bessel basis + polynomial envelope   mh1.cu:297-309, mh1_math.cuh:34-40
//   real spherical harmonics of -d (e3nn component norm)     mh1.cu:310-316, mh1_math.cuh:54-86
//   radial MLP with LayerNorm + SiLU and its r-tangent      mh1_math.cuh:121-173
//   radial projection x cutoff, density tanh(a^2) x cutoff   mh1.cu:331-368
//   channel-wise tensor-product messages                    mh1.cu:370-389
//   analytical backward: TP adjoints, r-tangent, forces     mh1.cu:390-452
//   ZBL pair repulsion                                      mh1.cu:471-537
// The B200 structure is different: edges are enumerated once per call into a CSR list,
// per-edge geometry and radial features are computed once per call (not per traversal),
// the tensor-product term table is compiled in so every accumulator lives in registers,
// forces are written per edge and gathered per atom through the reverse-edge index
// (deterministic, no force atomics), and per-atom sums are warp reductions.
#include "model.hpp"
#include "../lapis/launch.cuh"
#include "edge_common.cuh"
#include <type_traits>
#include <utility>

namespace mace {
using lapis::DeviceGeometry;
namespace {
using namespace edge;

// ---------------- ZBL (warp per receiver) ----------------
__global__ void zbl_kernel(DeviceGeometry g, const float *c, const float *radii, const float *coeff, float shift,
                           float *energy, float *force, float *virial) {
  int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (i >= g.n)
    return;
  float acc[13] = {};
  float zi = float(g.elements[i]);
  const float rates[4] = {3.2f, .9423f, .4028f, .2016f};
  for (int e = g.edge_offsets[i] + lane; e < g.edge_offsets[i + 1]; e += 32) {
    float4 d = g.edge_vector[e];
    float zj = float(g.elements[g.edge_sender[e]]);
    float r = d.w;
    if (r <= 0.f) {
      atomicCAS(g.status, 0, 1);
      continue;
    }
    float rc = radii[int(zi)] + radii[int(zj)];
    if (r >= rc)
      continue;
    D1 x{r, 1.f};
    float a = c[9] * .529f / (powf(zi, c[8]) + powf(zj, c[8]));
    D1 phi{0.f, 0.f};
#pragma unroll
    for (int t = 0; t < 4; ++t)
      phi = phi + cst(coeff[t]) * dexp(cst(-rates[t] / a) * x);
    D1 ev = cst(.5f * 14.3996f * zi * zj * c[6]) * phi / x * envelope(x, rc, c[10]);
    float v[3] = {d.x, d.y, d.z};
    acc[0] += ev.v;
#pragma unroll
    for (int k = 0; k < 3; ++k)
      acc[1 + k] += 2.f * ev.d * v[k] / r;
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
      for (int l = 0; l < 3; ++l)
        acc[4 + 3 * k + l] -= ev.d * v[k] * v[l] / r;
  }
#pragma unroll
  for (int q = 0; q < 13; ++q)
    acc[q] = warp_allsum(acc[q]);
  if (lane == 0) {
    energy[i] = shift + acc[0];
    for (int k = 0; k < 3; ++k)
      force[3 * i + k] = acc[1 + k];
    for (int k = 0; k < 9; ++k)
      virial[9 * i + k] = acc[4 + k];
  }
}

// ---------------- per-edge geometry (warp per receiver, lane per edge) ----------------
// A warp's 32 edges are one contiguous block of every per-edge array, so each lane writes its
// W values to its own padded shared-memory row (stride W + 1: conflict-free) and the warp
// then stores the block with consecutive lanes on consecutive floats.
constexpr int kGeometryThreads = 128, kGeometryRow = 49;

template <int W>
__device__ __forceinline__ void warp_rows_out(float *dst, const float (&v)[W], int cnt, int lane, float *buf) {
  static_assert(W + 1 <= kGeometryRow, "row buffer too small");
#pragma unroll
  for (int k = 0; k < W; ++k)
    buf[lane * (W + 1) + k] = v[k];
  __syncwarp();
  for (int f = lane; f < cnt * W; f += 32)
    dst[f] = buf[f + f / W];
  __syncwarp();
}

__global__ void __launch_bounds__(kGeometryThreads)
    geometry_kernel(DeviceGeometry g, const int *species, const float *c, const float *radii, const float *bessel,
                    EdgeArrays out, int *pair) {
  __shared__ float rows[kGeometryThreads / 32][32 * kGeometryRow];
  int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (i >= g.n)
    return;
  float *buf = rows[threadIdx.x >> 5];
  int zi = g.elements[i], si = species[i], end = g.edge_offsets[i + 1];
  for (int e0 = g.edge_offsets[i]; e0 < end; e0 += 32) {
    int e = e0 + lane, cnt = min(32, end - e0);
    bool valid = e < end;
    float4 d = valid ? g.edge_vector[e] : make_float4(0.f, 0.f, 1.f, 1.f);
    int j = valid ? g.edge_sender[e] : i;
    float r = d.w;
    if (r <= 0.f) {
      atomicCAS(g.status, 0, 1);
      r = 1e-10f;
    }
    int zj = g.elements[j];
    D1 dist{r, 1.f};
    D1 ratio = dist / cst(.5f * (radii[zj] + radii[zi]));
    D1 tr = cst(1.f) / (cst(1.f) + cst(c[3]) * dpow(ratio, c[4]) / (cst(1.f) + dpow(ratio, c[4] - c[5])));
    D1 cut = envelope(dist, c[0], c[2]);
    if (valid) {
      pair[e] = species[j] | (si << 16);
      out.cut[e] = make_float2(cut.v, cut.d);
    }
    float bv[10], bd[10];
#pragma unroll
    for (int k = 0; k < 10; ++k) {
      D1 b = cst(c[1]) * dsin(cst(bessel[k]) * tr) / tr;
      bv[k] = b.v;
      bd[k] = b.d;
    }
    warp_rows_out<10>(out.basis + size_t(e0) * 10, bv, cnt, lane, buf);
    warp_rows_out<10>(out.dbasis + size_t(e0) * 10, bd, cnt, lane, buf);
    float Y[16];
    if (out.dY) {
      float Gy[16][3];
      harmonics<true>(d.x, d.y, d.z, r, Y, Gy);
      warp_rows_out<48>(out.dY + size_t(e0) * 48, reinterpret_cast<const float(&)[48]>(Gy), cnt, lane, buf);
    } else {
      harmonics<false>(d.x, d.y, d.z, r, Y, nullptr);
    }
    warp_rows_out<16>(out.Y + size_t(e0) * 16, Y, cnt, lane, buf);
  }
}

// ---------------- radial MLP (register-tiled: 4 edges x 8 outputs per lane) ----------------
// The two 64 x 64 layers are small GEMMs over edges, fed from shared memory, which supplies one
// 32-lane word per clock against 128 FMA lanes: a lane therefore owns a 4-edge x 8-output tile
// (value and r-tangent, 64 accumulators), so every shared-memory word it loads feeds four FMAs.
// Lane = 8 * edge group + output group: the lane's edges are the warp's slots ge + 4 i (i < 4;
// interleaved so the four groups' rows fall on distinct banks) and its outputs
// u = 8 go .. 8 go + 7.  LayerNorm sums combine the 8 lanes of an edge group
// with three shuffles.  Weights and vectors are stored permuted ([k][go][12], 8 used) so the 8
// output groups of a quarter warp read distinct banks.  Each warp keeps its 16 edges' layer
// inputs in shared rows (value [0, 64), tangent [68, 132)) and their Bessel basis and
// r-derivative; a CTA of 16 warps (128 registers a thread) takes tiles of 256 edges.
struct RadialParams {
  Radial conv, dens;
};
constexpr int kRadialThreads = 512, kRadialWarps = kRadialThreads / 32, kRadialEdgesPerWarp = 16;
constexpr int kRadialEdges = kRadialWarps * kRadialEdgesPerWarp;
constexpr int kRadialRow = 132, kRadialTan = 68, kRadialBasis = 22; // basis, d basis / dr, cut pair
constexpr int kRadialPerm = 96; // floats per permuted 64-vector (8 groups x 12)
__host__ __device__ constexpr int radial_perm(int u) { return (u >> 3) * 12 + (u & 7); }
// Shared layout (floats): conv input [10][96], density input [10][96], W2 / W3 [64][96],
// 13 permuted vectors, then per warp: rows [16][132] and basis [16][22].
constexpr int kRadialIn = 10 * kRadialPerm, kRadialW = 64 * kRadialPerm, kRadialVecs = 13 * kRadialPerm;
constexpr int kRadialWarpFloats = kRadialEdgesPerWarp * (kRadialRow + kRadialBasis);
constexpr int kRadialSmemFloats = 2 * kRadialIn + 2 * kRadialW + kRadialVecs + kRadialWarps * kRadialWarpFloats;

// Sum over the 8 lanes of an edge group.
__device__ __forceinline__ float group_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v + __shfl_xor_sync(0xffffffffu, v, 4);
}

__device__ __forceinline__ void load8(const float *p, float (&v)[8]) {
  float4 x = *reinterpret_cast<const float4 *>(p), y = *reinterpret_cast<const float4 *>(p + 4);
  v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w, v[4] = y.x, v[5] = y.y, v[6] = y.z, v[7] = y.w;
}

// LayerNorm (biased variance, eps 1e-5) + SiLU with the forward tangent on the lane's 8
// outputs of edge i (statistics over the edge group's 8 lanes).
__device__ __forceinline__ void tile_ln_silu(float (&a)[8], float (&da)[8], const float *gamma, const float *beta) {
  float s = 0.f, d = 0.f;
#pragma unroll
  for (int m = 0; m < 8; ++m)
    s += a[m], d += da[m];
  float mean = group_sum(s) * (1.f / 64), dmean = group_sum(d) * (1.f / 64);
  float v = 0.f, c = 0.f;
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    a[m] -= mean;
    da[m] -= dmean;
    v = fmaf(a[m], a[m], v);
    c = fmaf(a[m], da[m], c);
  }
  float inv = rsqrtf(group_sum(v) * (1.f / 64) + 1e-5f);
  float dinv = -inv * inv * inv * group_sum(c) * (1.f / 64);
  float g[8], bt[8];
  load8(gamma, g);
  load8(beta, bt);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float x = a[m] * inv * g[m] + bt[m];
    float sg = sigm(x);
    float dx = (da[m] * inv + a[m] * dinv) * g[m];
    a[m] = x * sg;
    da[m] = dx * sg * (1.f + x * (1.f - sg));
  }
}

// Input layer for the lane's 4 edges: a = b0 + source[zs] + target[zr] + W1 x, da = W1 dx.
__device__ __forceinline__ void tile_input(float (&a)[4][8], float (&da)[4][8], const float *w1, const float *b0,
                                           const float *source, const float *target, const int (&zs)[4],
                                           const int (&zr)[4], int u0, const float *bas) { // bas: edge i at 4 i rows
  float b[8];
  load8(b0, b);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 *sp = reinterpret_cast<const float4 *>(source + zs[i] * 64 + u0);
    const float4 *tp = reinterpret_cast<const float4 *>(target + zr[i] * 64 + u0);
    float4 s0 = __ldg(sp), s1 = __ldg(sp + 1), t0 = __ldg(tp), t1 = __ldg(tp + 1);
    float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float tv[8] = {t0.x, t0.y, t0.z, t0.w, t1.x, t1.y, t1.z, t1.w};
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      a[i][m] = b[m] + sv[m] + tv[m];
      da[i][m] = 0.f;
    }
  }
#pragma unroll 2
  for (int k = 0; k < 10; ++k) {
    float w[8];
    load8(w1 + k * kRadialPerm, w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float xk = bas[4 * i * kRadialBasis + k], dxk = bas[4 * i * kRadialBasis + 10 + k];
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        a[i][m] = fmaf(w[m], xk, a[i][m]);
        da[i][m] = fmaf(w[m], dxk, da[i][m]);
      }
    }
  }
}

// The lane's outputs into its edges' rows (edge i at 4 i rows; after every lane of the warp has
// read them).
__device__ __forceinline__ void tile_store(float *rows, const float (&a)[4][8], const float (&da)[4][8], int u0) {
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float *r = rows + 4 * i * kRadialRow + u0;
    *reinterpret_cast<float4 *>(r) = make_float4(a[i][0], a[i][1], a[i][2], a[i][3]);
    *reinterpret_cast<float4 *>(r + 4) = make_float4(a[i][4], a[i][5], a[i][6], a[i][7]);
    *reinterpret_cast<float4 *>(r + kRadialTan) = make_float4(da[i][0], da[i][1], da[i][2], da[i][3]);
    *reinterpret_cast<float4 *>(r + kRadialTan + 4) = make_float4(da[i][4], da[i][5], da[i][6], da[i][7]);
  }
  __syncwarp();
}

// scaled: write cut h and cut dh + dcut h (the projection GEMM then yields w and its r-derivative
// directly); otherwise h and dh.
// One grid row (blockIdx.y) per layer: the layers' radial MLPs depend on the geometry only.
struct RadialLayers {
  RadialParams p[2];
  RadialOut o[2];
};
__global__ void __launch_bounds__(kRadialThreads, 1) radial_kernel(long long E, const __grid_constant__ RadialLayers RL,
                                                                const int *pair, EdgeArrays ea, int scaled) {
  const RadialParams &R = RL.p[blockIdx.y];
  const RadialOut &ro = RL.o[blockIdx.y];
  extern __shared__ __align__(16) float sm[];
  float *c_in = sm, *d_in = c_in + kRadialIn, *c_w = d_in + kRadialIn, *vecs = c_w + 2 * kRadialW;
  float *c_b = vecs, *c_g = vecs + 3 * kRadialPerm, *c_bt = vecs + 6 * kRadialPerm;
  float *d_b0 = vecs + 9 * kRadialPerm, *d_g = vecs + 10 * kRadialPerm, *d_bt = vecs + 11 * kRadialPerm;
  float *d_out = vecs + 12 * kRadialPerm;
  int t = threadIdx.x, lane = t & 31, warp = t >> 5, go = lane & 7, ge = lane >> 3;
  float *wrows = vecs + kRadialVecs + warp * kRadialWarpFloats;
  float *wbas = wrows + kRadialEdgesPerWarp * kRadialRow;
  for (int k = t; k < 640; k += kRadialThreads) {
    int o = (k >> 6) * kRadialPerm + radial_perm(k & 63);
    c_in[o] = R.conv.input_t[k];
    d_in[o] = R.dens.input_t[k];
  }
  for (int k = t; k < 4096; k += kRadialThreads) {
    int o = (k >> 6) * kRadialPerm + radial_perm(k & 63);
    c_w[o] = R.conv.weight_t[1][k];
    c_w[kRadialW + o] = R.conv.weight_t[2][k];
  }
  for (int k = t; k < 64; k += kRadialThreads) {
    int o = radial_perm(k);
    c_b[o] = R.conv.bias0[k];
    c_b[kRadialPerm + o] = R.conv.bias[1][k];
    c_b[2 * kRadialPerm + o] = R.conv.bias[2][k];
    for (int l = 0; l < 3; ++l) {
      c_g[l * kRadialPerm + o] = R.conv.gamma[l][k];
      c_bt[l * kRadialPerm + o] = R.conv.beta[l][k];
    }
    d_b0[o] = R.dens.bias0[k];
    d_g[o] = R.dens.gamma[0][k];
    d_bt[o] = R.dens.beta[0][k];
    d_out[o] = R.dens.out_t[k];
  }
  __syncthreads();
  const float d_ob = R.dens.out_b[0];
  const int u0 = 8 * go, po = go * 12; // the lane's outputs and their block in a permuted vector
  float *rows = wrows + ge * kRadialRow;
  const float *bas = wbas + ge * kRadialBasis;
  for (long long base = (long long)blockIdx.x * kRadialEdges; base < E; base += (long long)gridDim.x * kRadialEdges) {
    long long wbase = base + warp * kRadialEdgesPerWarp;
    int wcnt = E - wbase < kRadialEdgesPerWarp ? int(max(E - wbase, 0LL)) : kRadialEdgesPerWarp;
    // ---- the warp's 16 edges: Bessel basis and r-derivative into shared memory ----
    for (int f = lane; f < kRadialEdgesPerWarp * 10; f += 32) {
      int j = f / 10, k = f - 10 * j;
      bool ok = j < wcnt;
      wbas[j * kRadialBasis + k] = ok ? ea.basis[size_t(wbase) * 10 + f] : 0.f;
      wbas[j * kRadialBasis + 10 + k] = ok ? ea.dbasis[size_t(wbase) * 10 + f] : 0.f;
    }
    if (scaled && lane < kRadialEdgesPerWarp) {
      float2 cv = lane < wcnt ? ea.cut[wbase + lane] : make_float2(0.f, 0.f);
      wbas[lane * kRadialBasis + 20] = cv.x;
      wbas[lane * kRadialBasis + 21] = cv.y;
    }
    int zs[4], zr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int j = ge + 4 * i, p = j < wcnt ? pair[wbase + j] : 0;
      zs[i] = p & 0xffff, zr[i] = p >> 16;
    }
    __syncwarp();
    float a[4][8], da[4][8];
    // ---- conv radial network: 10 -> 64 -> 64 -> 64 ----
    tile_input(a, da, c_in + po, c_b + po, R.conv.source, R.conv.target, zs, zr, u0, bas);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      tile_ln_silu(a[i], da[i], c_g + po, c_bt + po);
    tile_store(rows, a, da, u0);
#pragma unroll 1
    for (int layer = 1; layer < 3; ++layer) {
      const float *W = c_w + (layer - 1) * kRadialW + po;
      float b[8];
      load8(c_b + layer * kRadialPerm + po, b);
      // Output pairs (2 p, 2 p + 1) accumulate with paired FMAs (fma.rn.f32x2: two IEEE FMAs).
      float2 a2[4][4], da2[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          a2[i][p] = make_float2(b[2 * p], b[2 * p + 1]);
          da2[i][p] = make_float2(0.f, 0.f);
        }
#pragma unroll 2
      for (int k = 0; k < 64; ++k) {
        const float4 *w4 = reinterpret_cast<const float4 *>(W + k * kRadialPerm);
        float4 wa = w4[0], wb = w4[1];
        float2 w2[4] = {make_float2(wa.x, wa.y), make_float2(wa.z, wa.w), make_float2(wb.x, wb.y),
                        make_float2(wb.z, wb.w)};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float hv = rows[4 * i * kRadialRow + k], dv = rows[4 * i * kRadialRow + kRadialTan + k];
          float2 h2 = make_float2(hv, hv), d2 = make_float2(dv, dv);
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            a2[i][p] = __ffma2_rn(w2[p], h2, a2[i][p]);
            da2[i][p] = __ffma2_rn(w2[p], d2, da2[i][p]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          a[i][2 * p] = a2[i][p].x, a[i][2 * p + 1] = a2[i][p].y;
          da[i][2 * p] = da2[i][p].x, da[i][2 * p + 1] = da2[i][p].y;
        }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        tile_ln_silu(a[i], da[i], c_g + layer * kRadialPerm + po, c_bt + layer * kRadialPerm + po);
      tile_store(rows, a, da, u0);
    }
    // ---- coalesced write of h / dh: the warp's 16 consecutive edges ----
#pragma unroll 4
    for (int f = lane; f < kRadialEdgesPerWarp * 64; f += 32) {
      int r = f >> 6, c = f & 63;
      if (r < wcnt) {
        size_t o = size_t(wbase) * 64 + f;
        float hv = wrows[r * kRadialRow + c], dv = wrows[r * kRadialRow + kRadialTan + c];
        if (scaled) {
          float cut = wbas[r * kRadialBasis + 20], dcut = wbas[r * kRadialBasis + 21];
          ro.h[o] = cut * hv;
          ro.dh[o] = fmaf(cut, dv, dcut * hv);
        } else {
          ro.h[o] = hv;
          ro.dh[o] = dv;
        }
      }
    }
    // ---- density network: 10 -> 64, LayerNorm + SiLU, -> 1, tanh(a^2) x cutoff ----
    tile_input(a, da, d_in + po, d_b0 + po, R.dens.source, R.dens.target, zs, zr, u0, bas);
    float ow[8];
    load8(d_out + po, ow);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      tile_ln_silu(a[i], da[i], d_g + po, d_bt + po);
      float sv = 0.f, dsv = 0.f;
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        sv = fmaf(ow[m], a[i][m], sv);
        dsv = fmaf(ow[m], da[i][m], dsv);
      }
      sv = group_sum(sv) + d_ob;
      dsv = group_sum(dsv);
      int j = ge + 4 * i;
      if (go == 0 && j < wcnt) {
        long long e = wbase + j;
        float2 cv = ea.cut[e];
        float den = tanhf(sv * sv);
        ro.density[e] = make_float2(den * cv.x, 2.f * sv * dsv * (1.f - den * den) * cv.x + den * cv.y);
      }
    }
    __syncwarp(); // rows and basis are rewritten by the next tile
  }
}

// ---------------- fused projection + tensor-product messages (CTA per receiver) ----------------
template <int L>
__global__ void __launch_bounds__(128) message_forward_kernel(int n, const int *row, const int *sender,
                                                              const float *h, const float *Y, const float2 *cut,
                                                              const float2 *den, const float *up,
                                                              const float *Wt, const float *Wb, TPValues cg,
                                                              float *msg, float *rho) {
  using T = Traits<L>;
  constexpr int P = T::P, NC = T::NC, IN = T::IN, EC = T::EC;
  __shared__ __align__(16) float hs[64][EC];
  __shared__ float ys[EC][16], cs[EC];
  __shared__ int js[EC];
  int i = blockIdx.x, c = threadIdx.x;
  float out[NC];
#pragma unroll
  for (int k = 0; k < NC; ++k)
    out[k] = 0.f;
  float bias[P];
#pragma unroll
  for (int p = 0; p < P; ++p)
    bias[p] = Wb[p * 128 + c];
  int begin = row[i], end = row[i + 1];
  for (int base = begin; base < end; base += EC) {
    int cnt = min(EC, end - base);
    for (int idx = c; idx < EC * 64; idx += 128) {
      int e = idx >> 6, a = idx & 63;
      hs[a][e] = e < cnt ? h[size_t(base + e) * 64 + a] : 0.f;
    }
    for (int idx = c; idx < EC * 16; idx += 128) {
      int e = idx >> 4, k = idx & 15;
      ys[e][k] = e < cnt ? Y[size_t(base + e) * 16 + k] : 0.f;
    }
    if (c < EC) {
      cs[c] = c < cnt ? cut[base + c].x : 0.f;
      js[c] = c < cnt ? sender[base + c] : 0;
    }
    __syncthreads();
    float acc[EC][P];
#pragma unroll
    for (int e = 0; e < EC; ++e)
#pragma unroll
      for (int p = 0; p < P; ++p)
        acc[e][p] = 0.f;
#pragma unroll 2
    for (int a = 0; a < 64; ++a) {
      float hv[EC];
#pragma unroll
      for (int e = 0; e < EC; e += 4) {
        float4 v = *reinterpret_cast<const float4 *>(&hs[a][e]);
        hv[e] = v.x, hv[e + 1] = v.y, hv[e + 2] = v.z, hv[e + 3] = v.w;
      }
#pragma unroll
      for (int p = 0; p < P; ++p) {
        float w = __ldg(Wt + a * (P * 128) + p * 128 + c);
#pragma unroll
        for (int e = 0; e < EC; ++e)
          acc[e][p] = fmaf(w, hv[e], acc[e][p]);
      }
    }
#pragma unroll
    for (int e = 0; e < EC; ++e) {
      if (e < cnt) {
        int j = js[e];
        float u[IN], w[P];
#pragma unroll
        for (int q = 0; q < IN; ++q)
          u[q] = up[(size_t(q) * n + j) * 128 + c];
#pragma unroll
        for (int p = 0; p < P; ++p)
          w[p] = cs[e] * (acc[e][p] + bias[p]);
        Unroll<0, T::NT>::run([&](auto tc) {
          constexpr int t = decltype(tc)::value;
          constexpr TPTerm q = T::term(t);
          out[q.out] = fmaf(cg.v[t] * ys[e][q.sh], u[q.in] * w[q.path], out[q.out]);
        });
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int k = 0; k < NC; ++k)
    msg[(size_t(k) * n + i) * 128 + c] = out[k];
  if (c == 0) {
    float s = 0.f;
    for (int e = begin; e < end; ++e)
      s += den[e].x;
    rho[i] = s;
  }
}

// ---------------- backward: TP adjoints, r-tangent, per-edge force ----------------
template <int L, bool Accumulate>
__global__ void __launch_bounds__(128) message_backward_kernel(
    int n, const int *row, const int *sender, const float4 *vec, const float *h, const float *dh, const float2 *cut,
    const float2 *den, const float *up, const float *Wt, const float *Wb, TPValues cg, const float *msg_grad,
    const float *rho_grad, float *ug_edge, float4 *edge_force) {
  using T = Traits<L>;
  constexpr int P = T::P, NC = T::NC, IN = T::IN, EC = T::EC;
  __shared__ __align__(16) float hs[64][EC];
  __shared__ __align__(16) float dhs[64][EC];
  __shared__ float ys[EC][16], gys[EC][16][3], red[4][EC][4];
  __shared__ float2 cs[EC];
  __shared__ float4 vd[EC];
  __shared__ float dd[EC];
  __shared__ int js[EC];
  int i = blockIdx.x, c = threadIdx.x, lane = c & 31, warp = c >> 5;
  float G[NC];
#pragma unroll
  for (int k = 0; k < NC; ++k)
    G[k] = msg_grad[(size_t(k) * n + i) * 128 + c];
  float rg = rho_grad[i];
  float bias[P];
#pragma unroll
  for (int p = 0; p < P; ++p)
    bias[p] = Wb[p * 128 + c];
  int begin = row[i], end = row[i + 1];
  for (int base = begin; base < end; base += EC) {
    int cnt = min(EC, end - base);
    for (int idx = c; idx < EC * 64; idx += 128) {
      int e = idx >> 6, a = idx & 63;
      bool ok = e < cnt;
      hs[a][e] = ok ? h[size_t(base + e) * 64 + a] : 0.f;
      dhs[a][e] = ok ? dh[size_t(base + e) * 64 + a] : 0.f;
    }
    if (c < EC) {
      int e = c;
      if (e < cnt) {
        float4 v = vec[base + e];
        float r = v.w > 0.f ? v.w : 1e-10f;
        float Yv[16], Gv[16][3];
        harmonics<true>(v.x, v.y, v.z, r, Yv, Gv);
        for (int k = 0; k < 16; ++k) {
          ys[e][k] = Yv[k];
          gys[e][k][0] = Gv[k][0];
          gys[e][k][1] = Gv[k][1];
          gys[e][k][2] = Gv[k][2];
        }
        vd[e] = make_float4(v.x, v.y, v.z, r);
        cs[e] = cut[base + e];
        dd[e] = den[base + e].y;
        js[e] = sender[base + e];
      }
    }
    __syncthreads();
    float aw[EC][P], ad[EC][P];
#pragma unroll
    for (int e = 0; e < EC; ++e)
#pragma unroll
      for (int p = 0; p < P; ++p)
        aw[e][p] = ad[e][p] = 0.f;
#pragma unroll 2
    for (int a = 0; a < 64; ++a) {
      float hv[EC], dv[EC];
#pragma unroll
      for (int e = 0; e < EC; e += 4) {
        float4 v = *reinterpret_cast<const float4 *>(&hs[a][e]);
        float4 d = *reinterpret_cast<const float4 *>(&dhs[a][e]);
        hv[e] = v.x, hv[e + 1] = v.y, hv[e + 2] = v.z, hv[e + 3] = v.w;
        dv[e] = d.x, dv[e + 1] = d.y, dv[e + 2] = d.z, dv[e + 3] = d.w;
      }
#pragma unroll
      for (int p = 0; p < P; ++p) {
        float w = __ldg(Wt + a * (P * 128) + p * 128 + c);
#pragma unroll
        for (int e = 0; e < EC; ++e) {
          aw[e][p] = fmaf(w, hv[e], aw[e][p]);
          ad[e][p] = fmaf(w, dv[e], ad[e][p]);
        }
      }
    }
#pragma unroll
    for (int e = 0; e < EC; ++e) {
      float dr = 0.f, gx = 0.f, gy = 0.f, gz = 0.f;
      if (e < cnt) {
        int j = js[e];
        float u[IN], w[P], dw[P], ug[IN];
#pragma unroll
        for (int q = 0; q < IN; ++q) {
          u[q] = up[(size_t(q) * n + j) * 128 + c];
          ug[q] = 0.f;
        }
        float2 cv = cs[e];
#pragma unroll
        for (int p = 0; p < P; ++p) {
          float s = aw[e][p] + bias[p];
          w[p] = cv.x * s;
          dw[p] = cv.x * ad[e][p] + cv.y * s;
        }
        Unroll<0, T::NT>::run([&](auto tc) {
          constexpr int t = decltype(tc)::value;
          constexpr TPTerm q = T::term(t);
          float av = G[q.out] * cg.v[t];
          float xv = av * u[q.in];
          float yv = ys[e][q.sh];
          dr = fmaf(xv * yv, dw[q.path], dr);
          float z = xv * w[q.path];
          gx = fmaf(z, gys[e][q.sh][0], gx);
          gy = fmaf(z, gys[e][q.sh][1], gy);
          gz = fmaf(z, gys[e][q.sh][2], gz);
          if constexpr (L > 0)
            ug[q.in] = fmaf(av * yv, w[q.path], ug[q.in]);
        });
        if constexpr (L > 0) {
#pragma unroll
          for (int q = 0; q < IN; ++q)
            ug_edge[(size_t(base + e) * IN + q) * 128 + c] = ug[q];
        }
      }
      dr = warp_allsum(dr);
      gx = warp_allsum(gx);
      gy = warp_allsum(gy);
      gz = warp_allsum(gz);
      if (lane == 0) {
        red[warp][e][0] = dr;
        red[warp][e][1] = gx;
        red[warp][e][2] = gy;
        red[warp][e][3] = gz;
      }
    }
    __syncthreads();
    if (c < cnt) {
      int e = c;
      float s[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        s[q] = red[0][e][q] + red[1][e][q] + red[2][e][q] + red[3][e][q];
      float4 v = vd[e];
      float dr = s[0] + rg * dd[e];
      float4 f = make_float4(s[1] + dr * v.x / v.w, s[2] + dr * v.y / v.w, s[3] + dr * v.z / v.w, 0.f);
      if (Accumulate) {
        float4 o = edge_force[base + e];
        f.x += o.x, f.y += o.y, f.z += o.z;
      }
      edge_force[base + e] = f;
    }
    __syncthreads();
  }
}

// Receiver force = sum of its edges' forces minus the reverse edges' forces (the reaction
// on the sender); virial = -sum d (x) f over the receiver's edges; plus the ZBL terms.
__global__ void force_gather_kernel(DeviceGeometry g, const float4 *ef, float *force, float *virial) {
  int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (i >= g.n)
    return;
  float acc[12] = {};
  for (int e = g.edge_offsets[i] + lane; e < g.edge_offsets[i + 1]; e += 32) {
    float4 f = ef[e], fr = ef[g.edge_reverse[e]], d = g.edge_vector[e];
    acc[0] += f.x - fr.x;
    acc[1] += f.y - fr.y;
    acc[2] += f.z - fr.z;
    float dv[3] = {d.x, d.y, d.z}, fv[3] = {f.x, f.y, f.z};
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int b = 0; b < 3; ++b)
        acc[3 + 3 * a + b] -= dv[a] * fv[b];
  }
#pragma unroll
  for (int q = 0; q < 12; ++q)
    acc[q] = warp_allsum(acc[q]);
  if (lane == 0) {
    for (int k = 0; k < 3; ++k)
      force[3 * i + k] += acc[k];
    for (int k = 0; k < 9; ++k)
      virial[9 * i + k] += acc[3 + k];
  }
}
// Domain form of force_gather_kernel: reverse edges outside the local graph (index < 0) are
// skipped -- their forces arrive from the ranks that own those receivers.
__global__ void force_gather_domain_kernel(DeviceGeometry g, const float4 *ef, float *force, float *virial) {
  int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (i >= g.n)
    return;
  float acc[12] = {};
  for (int e = g.edge_offsets[i] + lane; e < g.edge_offsets[i + 1]; e += 32) {
    float4 f = ef[e], d = g.edge_vector[e];
    int r = g.edge_reverse[e];
    float4 fr = r >= 0 ? ef[r] : make_float4(0.f, 0.f, 0.f, 0.f);
    acc[0] += f.x - fr.x;
    acc[1] += f.y - fr.y;
    acc[2] += f.z - fr.z;
    float dv[3] = {d.x, d.y, d.z}, fv[3] = {f.x, f.y, f.z};
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int b = 0; b < 3; ++b)
        acc[3 + 3 * a + b] -= dv[a] * fv[b];
  }
#pragma unroll
  for (int q = 0; q < 12; ++q)
    acc[q] = warp_allsum(acc[q]);
  if (lane == 0) {
    for (int k = 0; k < 3; ++k)
      force[3 * i + k] += acc[k];
    for (int k = 0; k < 9; ++k)
      virial[9 * i + k] += acc[3 + k];
  }
}
} // namespace

void launch_force_gather_domain(cudaStream_t s, const DeviceGeometry &g, const float4 *edge_force, float *force,
                                float *virial) {
  if (g.n && g.edge_capacity)
    lapis::launch(force_gather_domain_kernel, (g.n * 32 + 255) / 256, 256, 0, s, g, edge_force, force, virial);
}

void launch_zbl(cudaStream_t s, const DeviceGeometry &g, const float *constants, const float *radii,
                const float *coeff, float shift, float *energy, float *force, float *virial) {
  if (g.n)
    lapis::launch(zbl_kernel, (g.n * 32 + 255) / 256, 256, 0, s, g, constants, radii, coeff, shift, energy, force, virial);
}

void launch_edge_geometry(cudaStream_t s, const DeviceGeometry &g, const int *species, const float *constants,
                          const float *radii, const float *bessel, EdgeArrays ea, int *pair) {
  if (g.n)
    lapis::launch(geometry_kernel, (g.n * 32 + kGeometryThreads - 1) / kGeometryThreads, kGeometryThreads, 0, s, g,
                  species, constants, radii, bessel, ea, pair);
}

void launch_radial(cudaStream_t s, const DeviceGeometry &g, const Layer *const *layers, const RadialOut *ro,
                   int count, const int *pair, EdgeArrays ea, bool scaled) {
  long long E = g.edge_capacity;
  if (!E || count < 1)
    return;
  if (count > 2)
    throw lapis::Error("launch_radial: at most two layers per launch");
  size_t smem = kRadialSmemFloats * sizeof(float);
  lapis::check(cudaFuncSetAttribute(radial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  RadialLayers rl{};
  for (int k = 0; k < count; ++k) {
    rl.p[k] = RadialParams{layers[k]->radial, layers[k]->density};
    rl.o[k] = ro[k];
  }
  long long tiles = (E + kRadialEdges - 1) / kRadialEdges;
  dim3 grid(unsigned(std::min<long long>(tiles, 148 * 2 / count)), unsigned(count));
  lapis::launch(radial_kernel, grid, kRadialThreads, smem, s, E, rl, pair, ea, int(scaled));
}

void launch_message_forward(cudaStream_t s, int layer, const DeviceGeometry &g, const Layer &l, EdgeArrays ea,
                            RadialOut ro, const float *up, float *message, float *density) {
  if (!g.n)
    return;
  if (layer == 0)
    lapis::launch(message_forward_kernel<0>, g.n, 128, 0, s, g.n, g.edge_offsets, g.edge_sender, ro.h, ea.Y, ea.cut, ro.density,
                                                  up, l.radial.out_t, l.radial.out_b, l.tp, message, density);
  else
    lapis::launch(message_forward_kernel<1>, g.n, 128, 0, s, g.n, g.edge_offsets, g.edge_sender, ro.h, ea.Y, ea.cut, ro.density,
                                                  up, l.radial.out_t, l.radial.out_b, l.tp, message, density);
}

void launch_message_backward(cudaStream_t s, int layer, const DeviceGeometry &g, const Layer &l, EdgeArrays ea,
                             RadialOut ro, const float *up, const float *message_grad, const float *density_grad,
                             float *ug_edge, float4 *edge_force, bool accumulate) {
  if (!g.n)
    return;
#define MH1_BWD(L, A)                                                                                              \
  lapis::launch(message_backward_kernel<L, A>, g.n, 128, 0, s, g.n, g.edge_offsets, g.edge_sender, g.edge_vector, ro.h, ro.dh, \
                                                    ea.cut, ro.density, up, l.radial.out_t, l.radial.out_b, l.tp,  \
                                                    message_grad, density_grad, ug_edge, edge_force)
  if (layer == 0) {
    if (accumulate)
      MH1_BWD(0, true);
    else
      MH1_BWD(0, false);
  } else {
    if (accumulate)
      MH1_BWD(1, true);
    else
      MH1_BWD(1, false);
  }
#undef MH1_BWD
}

void launch_force_gather(cudaStream_t s, const DeviceGeometry &g, const float4 *edge_force, float *force,
                         float *virial) {
  if (g.n && g.edge_capacity)
    lapis::launch(force_gather_kernel, (g.n * 32 + 255) / 256, 256, 0, s, g, edge_force, force, virial);
}
} // namespace mace
