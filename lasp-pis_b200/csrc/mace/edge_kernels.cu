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

// ---------------- radial MLP (warp per group of 4 edges) ----------------
struct RadialParams {
  Radial conv, dens;
};
// Shared layout: conv input [10][64], conv W1/W2 [64][64], density input [10][64], 13 x 64
// vectors (biases, gammas, betas, density output), then per-warp staging [2][64][4].
constexpr int kRadialSmemFloats = 640 + 2 * 4096 + 640 + 13 * 64 + 4 * 2 * 64 * 4;

// LayerNorm (biased variance, eps 1e-5) + SiLU with its tangent, for 4 edges in a warp;
// lane holds units lane and lane + 32.
__device__ __forceinline__ void ln_silu(float (&a)[4][2], float (&da)[4][2], const float *gamma,
                                        const float *beta, int lane) {
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float mean = warp_allsum(a[e][0] + a[e][1]) * (1.f / 64);
    float dmean = warp_allsum(da[e][0] + da[e][1]) * (1.f / 64);
    a[e][0] -= mean, a[e][1] -= mean;
    da[e][0] -= dmean, da[e][1] -= dmean;
    float inv = rsqrtf(warp_allsum(a[e][0] * a[e][0] + a[e][1] * a[e][1]) * (1.f / 64) + 1e-5f);
    float dinv = -inv * inv * inv * warp_allsum(a[e][0] * da[e][0] + a[e][1] * da[e][1]) * (1.f / 64);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      int t = lane + 32 * q;
      float u = a[e][q] * inv * gamma[t] + beta[t];
      float s = sigm(u);
      float du = (da[e][q] * inv + a[e][q] * dinv) * gamma[t];
      a[e][q] = u * s;
      da[e][q] = du * s * (1.f + u * (1.f - s));
    }
  }
}

__global__ void __launch_bounds__(128) radial_kernel(long long E, RadialParams R, const int *pair,
                                                     EdgeArrays ea, RadialOut ro) {
  extern __shared__ float sm[];
  float *c_in = sm, *c_w1 = c_in + 640, *c_w2 = c_w1 + 4096, *d_in = c_w2 + 4096, *misc = d_in + 640;
  float *c_b0 = misc, *c_b1 = misc + 64, *c_b2 = misc + 128, *d_b0 = misc + 192, *d_out = misc + 256;
  float *c_g = misc + 320, *c_bt = c_g + 192, *d_g = c_bt + 192, *d_bt = d_g + 64;
  float *stage = d_bt + 64; // [warp][2][64][4]
  int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  for (int k = t; k < 640; k += 128) {
    c_in[k] = R.conv.input_t[k];
    d_in[k] = R.dens.input_t[k];
  }
  for (int k = t; k < 4096; k += 128) {
    c_w1[k] = R.conv.weight_t[1][k];
    c_w2[k] = R.conv.weight_t[2][k];
  }
  for (int k = t; k < 64; k += 128) {
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
  float4 *hs = reinterpret_cast<float4 *>(stage + warp * 512), *dhs = hs + 64;
  long long groups = (E + 3) / 4;
  for (long long grp = blockIdx.x * 4ll + warp; grp < groups; grp += gridDim.x * 4ll) {
    long long e0 = grp * 4;
    int zs[4], zr[4];
    float x[4][10], dx[4][10], cutv[4][2];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      bool ok = e0 + e < E;
      int p = ok ? pair[e0 + e] : 0;
      zs[e] = p & 0xffff;
      zr[e] = p >> 16;
      float2 cv = ok ? ea.cut[e0 + e] : make_float2(0.f, 0.f);
      cutv[e][0] = cv.x;
      cutv[e][1] = cv.y;
#pragma unroll
      for (int k = 0; k < 10; ++k) {
        x[e][k] = ok ? ea.basis[(e0 + e) * 10 + k] : 0.f;
        dx[e][k] = ok ? ea.dbasis[(e0 + e) * 10 + k] : 0.f;
      }
    }
    // ---- conv radial network: 10 -> 64 -> 64 -> 64 ----
    float a[4][2], da[4][2];
#pragma unroll
    for (int e = 0; e < 4; ++e)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        int u = lane + 32 * q;
        float s = c_b0[u] + R.conv.source[zs[e] * 64 + u] + R.conv.target[zr[e] * 64 + u], ds = 0.f;
#pragma unroll
        for (int k = 0; k < 10; ++k) {
          float w = c_in[k * 64 + u];
          s = fmaf(w, x[e][k], s);
          ds = fmaf(w, dx[e][k], ds);
        }
        a[e][q] = s;
        da[e][q] = ds;
      }
    ln_silu(a, da, c_g, c_bt, lane);
#pragma unroll
    for (int layer = 1; layer < 3; ++layer) {
      const float *W = layer == 1 ? c_w1 : c_w2, *bias = layer == 1 ? c_b1 : c_b2;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        int u = lane + 32 * q;
        hs[u] = make_float4(a[0][q], a[1][q], a[2][q], a[3][q]);
        dhs[u] = make_float4(da[0][q], da[1][q], da[2][q], da[3][q]);
      }
      __syncwarp();
      float b0 = bias[lane], b1 = bias[lane + 32];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        a[e][0] = b0, a[e][1] = b1;
        da[e][0] = da[e][1] = 0.f;
      }
#pragma unroll 8
      for (int k = 0; k < 64; ++k) {
        float4 hv = hs[k], dv = dhs[k];
        float w0 = W[k * 64 + lane], w1 = W[k * 64 + lane + 32];
        float hv4[4] = {hv.x, hv.y, hv.z, hv.w}, dv4[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          a[e][0] = fmaf(w0, hv4[e], a[e][0]);
          a[e][1] = fmaf(w1, hv4[e], a[e][1]);
          da[e][0] = fmaf(w0, dv4[e], da[e][0]);
          da[e][1] = fmaf(w1, dv4[e], da[e][1]);
        }
      }
      __syncwarp();
      ln_silu(a, da, c_g + layer * 64, c_bt + layer * 64, lane);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (e0 + e < E)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          ro.h[(e0 + e) * 64 + lane + 32 * q] = a[e][q];
          ro.dh[(e0 + e) * 64 + lane + 32 * q] = da[e][q];
        }
    // ---- density network: 10 -> 64, LayerNorm + SiLU, -> 1, tanh(a^2) x cutoff ----
#pragma unroll
    for (int e = 0; e < 4; ++e)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        int u = lane + 32 * q;
        float s = d_b0[u] + R.dens.source[zs[e] * 64 + u] + R.dens.target[zr[e] * 64 + u], ds = 0.f;
#pragma unroll
        for (int k = 0; k < 10; ++k) {
          float w = d_in[k * 64 + u];
          s = fmaf(w, x[e][k], s);
          ds = fmaf(w, dx[e][k], ds);
        }
        a[e][q] = s;
        da[e][q] = ds;
      }
    ln_silu(a, da, d_g, d_bt, lane);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float s = warp_allsum(d_out[lane] * a[e][0] + d_out[lane + 32] * a[e][1]) + d_ob;
      float ds = warp_allsum(d_out[lane] * da[e][0] + d_out[lane + 32] * da[e][1]);
      if (lane == 0 && e0 + e < E) {
        float den = tanhf(s * s);
        ro.density[e0 + e] =
            make_float2(den * cutv[e][0], 2.f * s * ds * (1.f - den * den) * cutv[e][0] + den * cutv[e][1]);
      }
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
} // namespace

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
  long long groups = (E + 3) / 4;
  int blocks = int(std::min<long long>((groups + 3) / 4, 148 * 8));
  lapis::launch(radial_kernel, blocks, 128, smem, s, E, RadialParams{l.radial, l.density}, pair, ea, ro);
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
