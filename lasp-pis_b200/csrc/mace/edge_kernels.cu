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
__global__ void geometry_kernel(DeviceGeometry g, const int *species, const float *c, const float *radii,
                                const float *bessel, EdgeArrays out, int *pair) {
  int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (i >= g.n)
    return;
  int zi = g.elements[i], si = species[i];
  for (int e = g.edge_offsets[i] + lane; e < g.edge_offsets[i + 1]; e += 32) {
    int j = g.edge_sender[e];
    float4 d = g.edge_vector[e];
    float r = d.w;
    if (r <= 0.f) {
      atomicCAS(g.status, 0, 1);
      r = 1e-10f;
    }
    int zj = g.elements[j];
    pair[e] = species[j] | (si << 16);
    D1 dist{r, 1.f};
    D1 ratio = dist / cst(.5f * (radii[zj] + radii[zi]));
    D1 tr = cst(1.f) / (cst(1.f) + cst(c[3]) * dpow(ratio, c[4]) / (cst(1.f) + dpow(ratio, c[4] - c[5])));
    D1 cut = envelope(dist, c[0], c[2]);
    out.cut[e] = make_float2(cut.v, cut.d);
#pragma unroll
    for (int k = 0; k < 10; ++k) {
      D1 b = cst(c[1]) * dsin(cst(bessel[k]) * tr) / tr;
      out.basis[size_t(e) * 10 + k] = b.v;
      out.dbasis[size_t(e) * 10 + k] = b.d;
    }
    float Y[16];
    if (out.dY) {
      float Gy[16][3];
      harmonics<true>(d.x, d.y, d.z, r, Y, Gy);
#pragma unroll
      for (int k = 0; k < 16; ++k)
#pragma unroll
        for (int q = 0; q < 3; ++q)
          out.dY[size_t(e) * 48 + 3 * k + q] = Gy[k][q];
    } else {
      harmonics<false>(d.x, d.y, d.z, r, Y, nullptr);
    }
#pragma unroll
    for (int k = 0; k < 16; ++k)
      out.Y[size_t(e) * 16 + k] = Y[k];
  }
}

// ---------------- radial MLP (thread per edge) ----------------
// Each thread owns one edge.  A layer's 64 outputs and their r-tangents accumulate in
// registers from warp-wide broadcast float4 weight reads, then go to the thread's own padded
// shared-memory row (stride 65: conflict-free), where LayerNorm (in-thread sums) and SiLU
// run as rolled loops -- keeping the kernel small enough for the instruction cache -- and
// leave the next layer's input in place.  The final rows are written out coalesced.
struct RadialParams {
  Radial conv, dens;
};
constexpr int kRadialThreads = 128, kRadialRow = 65;
// Shared layout (floats): conv input [10][64], W2 / W3 [64 in][64 out], density input
// [10][64], 13 vectors of 64, then per-thread rows [128][2][65] (value, tangent).
constexpr int kRadialSmemFloats = 640 + 2 * 4096 + 640 + 13 * 64 + kRadialThreads * 2 * kRadialRow;

// Store accumulators to the row, then LayerNorm (biased variance, eps 1e-5) + SiLU with the
// forward tangent, in place.
__device__ __forceinline__ void row_ln_silu(const float (&a)[64], const float (&da)[64], float *row, float *drow,
                                            const float *gamma, const float *beta) {
  float s0 = 0.f, s1 = 0.f, d0 = 0.f, d1 = 0.f;
#pragma unroll
  for (int u = 0; u < 64; u += 2) {
    row[u] = a[u], row[u + 1] = a[u + 1];
    drow[u] = da[u], drow[u + 1] = da[u + 1];
    s0 += a[u], s1 += a[u + 1];
    d0 += da[u], d1 += da[u + 1];
  }
  float mean = (s0 + s1) * (1.f / 64), dmean = (d0 + d1) * (1.f / 64);
  float v0 = 0.f, v1 = 0.f, c0 = 0.f, c1 = 0.f;
#pragma unroll 4
  for (int u = 0; u < 64; u += 2) {
    float x0 = row[u] - mean, x1 = row[u + 1] - mean;
    float t0 = drow[u] - dmean, t1 = drow[u + 1] - dmean;
    v0 = fmaf(x0, x0, v0), v1 = fmaf(x1, x1, v1);
    c0 = fmaf(x0, t0, c0), c1 = fmaf(x1, t1, c1);
  }
  float inv = rsqrtf((v0 + v1) * (1.f / 64) + 1e-5f);
  float dinv = -inv * inv * inv * (c0 + c1) * (1.f / 64);
#pragma unroll 2
  for (int u = 0; u < 64; ++u) {
    float xc = row[u] - mean, tc = drow[u] - dmean;
    float x = xc * inv * gamma[u] + beta[u];
    float sg = sigm(x);
    float dx = (tc * inv + xc * dinv) * gamma[u];
    row[u] = x * sg;
    drow[u] = dx * sg * (1.f + x * (1.f - sg));
  }
}

// First layer: a = b0 + source[zs] + target[zr] + W1 x, da = W1 dx.
__device__ __forceinline__ void radial_input(float (&a)[64], float (&da)[64], const float *w1, const float *b0,
                                             const float *source, const float *target, int zs, int zr,
                                             const float (&x)[10], const float (&dx)[10]) {
  const float4 *src = reinterpret_cast<const float4 *>(source + zs * 64);
  const float4 *tgt = reinterpret_cast<const float4 *>(target + zr * 64);
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    float4 sv = __ldg(src + q), tv = __ldg(tgt + q);
    a[4 * q] = b0[4 * q] + sv.x + tv.x;
    a[4 * q + 1] = b0[4 * q + 1] + sv.y + tv.y;
    a[4 * q + 2] = b0[4 * q + 2] + sv.z + tv.z;
    a[4 * q + 3] = b0[4 * q + 3] + sv.w + tv.w;
    da[4 * q] = da[4 * q + 1] = da[4 * q + 2] = da[4 * q + 3] = 0.f;
  }
#pragma unroll 1
  for (int k = 0; k < 10; ++k) {
    const float4 *w = reinterpret_cast<const float4 *>(w1 + k * 64);
    float xk = x[k], dxk = dx[k];
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      float4 wv = w[q];
      a[4 * q] = fmaf(wv.x, xk, a[4 * q]);
      a[4 * q + 1] = fmaf(wv.y, xk, a[4 * q + 1]);
      a[4 * q + 2] = fmaf(wv.z, xk, a[4 * q + 2]);
      a[4 * q + 3] = fmaf(wv.w, xk, a[4 * q + 3]);
      da[4 * q] = fmaf(wv.x, dxk, da[4 * q]);
      da[4 * q + 1] = fmaf(wv.y, dxk, da[4 * q + 1]);
      da[4 * q + 2] = fmaf(wv.z, dxk, da[4 * q + 2]);
      da[4 * q + 3] = fmaf(wv.w, dxk, da[4 * q + 3]);
    }
  }
}

__global__ void __launch_bounds__(kRadialThreads) radial_kernel(long long E, RadialParams R, const int *pair,
                                                                EdgeArrays ea, RadialOut ro) {
  extern __shared__ float sm[];
  float *c_in = sm, *c_w1 = c_in + 640, *c_w2 = c_w1 + 4096, *d_in = c_w2 + 4096, *vecs = d_in + 640;
  float *c_b0 = vecs, *c_b1 = vecs + 64, *c_b2 = vecs + 128, *d_b0 = vecs + 192, *d_out = vecs + 256;
  float *c_g = vecs + 320, *c_bt = c_g + 192, *d_g = c_bt + 192, *d_bt = d_g + 64;
  float *rows = vecs + 13 * 64;
  int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  for (int k = t; k < 640; k += kRadialThreads) {
    c_in[k] = R.conv.input_t[k];
    d_in[k] = R.dens.input_t[k];
  }
  for (int k = t; k < 4096; k += kRadialThreads) {
    c_w1[k] = R.conv.weight_t[1][k];
    c_w2[k] = R.conv.weight_t[2][k];
  }
  for (int k = t; k < 64; k += kRadialThreads) {
    c_b0[k] = R.conv.bias0[k];
    c_b1[k] = R.conv.bias[1][k];
    c_b2[k] = R.conv.bias[2][k];
    d_b0[k] = R.dens.bias0[k];
    d_out[k] = R.dens.out_t[k];
    for (int l = 0; l < 3; ++l) {
      c_g[l * 64 + k] = R.conv.gamma[l][k];
      c_bt[l * 64 + k] = R.conv.beta[l][k];
    }
    d_g[k] = R.dens.gamma[0][k];
    d_bt[k] = R.dens.beta[0][k];
  }
  __syncthreads();
  float d_ob = R.dens.out_b[0];
  float *my = rows + t * 2 * kRadialRow, *my_d = my + kRadialRow;
  for (long long base = (long long)blockIdx.x * kRadialThreads; base < E; base += (long long)gridDim.x * kRadialThreads) {
    long long e = base + t;
    bool ok = e < E;
    int p = ok ? pair[e] : 0, zs = p & 0xffff, zr = p >> 16;
    float x[10], dx[10];
#pragma unroll
    for (int k = 0; k < 10; ++k) {
      x[k] = ok ? ea.basis[e * 10 + k] : 0.f;
      dx[k] = ok ? ea.dbasis[e * 10 + k] : 0.f;
    }
    float2 cv = ok ? ea.cut[e] : make_float2(0.f, 0.f);
    float a[64], da[64];
    // ---- conv radial network: 10 -> 64 -> 64 -> 64 ----
    radial_input(a, da, c_in, c_b0, R.conv.source, R.conv.target, zs, zr, x, dx);
    row_ln_silu(a, da, my, my_d, c_g, c_bt);
#pragma unroll 1
    for (int layer = 1; layer < 3; ++layer) {
      const float *W = layer == 1 ? c_w1 : c_w2, *bias = layer == 1 ? c_b1 : c_b2;
#pragma unroll
      for (int u = 0; u < 64; ++u) {
        a[u] = bias[u];
        da[u] = 0.f;
      }
#pragma unroll 1
      for (int k = 0; k < 64; ++k) {
        float hv = my[k], dv = my_d[k];
        const float4 *w = reinterpret_cast<const float4 *>(W + k * 64);
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          float4 wv = w[q];
          a[4 * q] = fmaf(wv.x, hv, a[4 * q]);
          a[4 * q + 1] = fmaf(wv.y, hv, a[4 * q + 1]);
          a[4 * q + 2] = fmaf(wv.z, hv, a[4 * q + 2]);
          a[4 * q + 3] = fmaf(wv.w, hv, a[4 * q + 3]);
          da[4 * q] = fmaf(wv.x, dv, da[4 * q]);
          da[4 * q + 1] = fmaf(wv.y, dv, da[4 * q + 1]);
          da[4 * q + 2] = fmaf(wv.z, dv, da[4 * q + 2]);
          da[4 * q + 3] = fmaf(wv.w, dv, da[4 * q + 3]);
        }
      }
      row_ln_silu(a, da, my, my_d, c_g + layer * 64, c_bt + layer * 64);
    }
    // ---- coalesced write of h / dh: 32 consecutive edges per warp ----
    __syncwarp();
    long long wbase = base + warp * 32;
    const float *wrows = rows + warp * 32 * 2 * kRadialRow;
#pragma unroll 1
    for (int r = 0; r < 32 && wbase + r < E; ++r) {
      const float *src = wrows + r * 2 * kRadialRow;
      size_t o = size_t(wbase + r) * 64;
      ro.h[o + lane] = src[lane];
      ro.h[o + 32 + lane] = src[32 + lane];
      ro.dh[o + lane] = src[kRadialRow + lane];
      ro.dh[o + 32 + lane] = src[kRadialRow + 32 + lane];
    }
    __syncwarp();
    // ---- density network: 10 -> 64, LayerNorm + SiLU, -> 1, tanh(a^2) x cutoff ----
    radial_input(a, da, d_in, d_b0, R.dens.source, R.dens.target, zs, zr, x, dx);
    row_ln_silu(a, da, my, my_d, d_g, d_bt);
    float sv = d_ob, dsv = 0.f;
#pragma unroll 4
    for (int u = 0; u < 64; ++u) {
      sv = fmaf(d_out[u], my[u], sv);
      dsv = fmaf(d_out[u], my_d[u], dsv);
    }
    __syncwarp();
    if (ok) {
      float den = tanhf(sv * sv);
      ro.density[e] = make_float2(den * cv.x, 2.f * sv * dsv * (1.f - den * den) * cv.x + den * cv.y);
    }
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
    const float *rho_grad, float *up_grad, float4 *edge_force) {
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
            atomicAdd(up_grad + (size_t(q) * n + j) * 128 + c, ug[q]);
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
// The reaction of every local edge on a ghost sender, accumulated in the ghost's force row.
__global__ void ghost_reaction_kernel(long long E, int n_own, const int *sender, const float4 *ef, float *force) {
  long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (e >= E)
    return;
  int j = sender[e];
  if (j >= n_own) {
    float4 f = ef[e];
    atomicAdd(force + 3 * j, -f.x);
    atomicAdd(force + 3 * j + 1, -f.y);
    atomicAdd(force + 3 * j + 2, -f.z);
  }
}
} // namespace

void launch_force_gather_domain(cudaStream_t s, const DeviceGeometry &g, const float4 *edge_force, float *force,
                                float *virial) {
  if (g.n && g.edge_capacity)
    lapis::launch(force_gather_domain_kernel, (g.n * 32 + 255) / 256, 256, 0, s, g, edge_force, force, virial);
  if (g.edge_capacity)
    lapis::launch(ghost_reaction_kernel, int((g.edge_capacity + 255) / 256), 256, 0, s, g.edge_capacity, g.n,
                  g.edge_sender, edge_force, force);
}

void launch_zbl(cudaStream_t s, const DeviceGeometry &g, const float *constants, const float *radii,
                const float *coeff, float shift, float *energy, float *force, float *virial) {
  if (g.n)
    lapis::launch(zbl_kernel, (g.n * 32 + 255) / 256, 256, 0, s, g, constants, radii, coeff, shift, energy, force, virial);
}

void launch_edge_geometry(cudaStream_t s, const DeviceGeometry &g, const int *species, const float *constants,
                          const float *radii, const float *bessel, EdgeArrays ea, int *pair) {
  if (g.n)
    lapis::launch(geometry_kernel, (g.n * 32 + 255) / 256, 256, 0, s, g, species, constants, radii, bessel, ea, pair);
}

void launch_radial(cudaStream_t s, const DeviceGeometry &g, const Layer &l, const int *pair, EdgeArrays ea,
                   RadialOut ro) {
  long long E = g.edge_capacity;
  if (!E)
    return;
  size_t smem = kRadialSmemFloats * sizeof(float);
  lapis::check(cudaFuncSetAttribute(radial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  long long tiles = (E + kRadialThreads - 1) / kRadialThreads;
  int blocks = int(std::min<long long>(tiles, 148 * 2));
  lapis::launch(radial_kernel, blocks, kRadialThreads, smem, s, E, RadialParams{l.radial, l.density}, pair, ea, ro);
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
                             float *up_grad, float4 *edge_force, bool accumulate) {
  if (!g.n)
    return;
#define MH1_BWD(L, A)                                                                                              \
  lapis::launch(message_backward_kernel<L, A>, g.n, 128, 0, s, g.n, g.edge_offsets, g.edge_sender, g.edge_vector, ro.h, ro.dh, \
                                                    ea.cut, ro.density, up, l.radial.out_t, l.radial.out_b, l.tp,  \
                                                    message_grad, density_grad, up_grad, edge_force)
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
