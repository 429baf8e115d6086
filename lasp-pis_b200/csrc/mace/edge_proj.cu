// Edge tensor-product kernels over a precomputed radial projection.
//
// The radial projection of the reference's MH1Pair (mace/src/mh1.cu:331-353),
//     R[e][p*128 + c] = sum_a h[e][a] W[a][p*128 + c]        (and dR from dh/dr),
// is one dense E x 64 x (P*128) GEMM per layer.  Here it runs on the tensor cores (tc_gemm,
// tf32 hi/lo split with FP32 drains) into an HBM buffer, chunked by receivers, and the
// kernels below consume it:
//   forward   messages and density, as mace/src/mh1.cu:331-389 (w = cut * (R + b));
//   backward  tensor-product adjoints, r-tangent and per-edge force, as mh1.cu:390-452.
// The backward regroups the term sum so that each term costs six FP32 operations: per path
// Q_p = sum_t cg G[out] u[in] Y[sh] (then dE/dr = sum_p Q_p dw_p), per harmonic
// T_sh = sum_t cg G[out] u[in] w_p (then dE/dd = sum_sh T_sh dY_sh), and the sender
// up-gradient sum_t cg G[out] Y[sh] w_p.  dY comes precomputed from the geometry kernel.
// CTA per receiver, thread per channel; per-edge scalars are reduced over the 128 channels
// with warp shuffles and a 4-warp shared-memory sum in a fixed order.
#include "../lapis/launch.cuh"
#include "edge_common.cuh"
#include "model.hpp"

namespace mace {
using lapis::DeviceGeometry;
namespace {
using namespace edge;

template <int L>
__global__ void __launch_bounds__(128) message_forward_proj_kernel(int n, int r0, int e_base, const int *row,
                                                                   const int *sender, const float *R,
                                                                   const float *Y, const float2 *cut,
                                                                   const float2 *den, const float *up,
                                                                   const float *Wb, TPValues cg, float *msg,
                                                                   float *rho) {
  using T = Traits<L>;
  constexpr int P = T::P, NC = T::NC, IN = T::IN;
  int i = r0 + blockIdx.x, c = threadIdx.x;
  float out[NC];
#pragma unroll
  for (int k = 0; k < NC; ++k)
    out[k] = 0.f;
  float bias[P];
#pragma unroll
  for (int p = 0; p < P; ++p)
    bias[p] = Wb[p * 128 + c];
  int begin = row[i], end = row[i + 1];
  float rsum = 0.f;
#pragma unroll 1
  for (int e = begin; e < end; ++e) {
    const float *Re = R + size_t(e - e_base) * (P * 128) + c;
    float rv[P];
#pragma unroll
    for (int p = 0; p < P; ++p)
      rv[p] = __ldcs(Re + p * 128);
    int j = __ldg(sender + e);
    float cv = __ldg(&cut[e].x);
    float u[IN];
#pragma unroll
    for (int q = 0; q < IN; ++q)
      u[q] = __ldg(up + (size_t(q) * n + j) * 128 + c);
    float y[16];
    const float4 *y4 = reinterpret_cast<const float4 *>(Y + size_t(e) * 16);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float4 v = __ldg(y4 + k);
      y[4 * k] = v.x, y[4 * k + 1] = v.y, y[4 * k + 2] = v.z, y[4 * k + 3] = v.w;
    }
    float w[P];
#pragma unroll
    for (int p = 0; p < P; ++p)
      w[p] = cv * (rv[p] + bias[p]);
    Unroll<0, T::NT>::run([&](auto tc) {
      constexpr int t = decltype(tc)::value;
      constexpr TPTerm q = T::term(t);
      out[q.out] = fmaf(cg.v[t] * y[q.sh], u[q.in] * w[q.path], out[q.out]);
    });
    if (c == 0)
      rsum += den[e].x;
  }
#pragma unroll
  for (int k = 0; k < NC; ++k)
    msg[(size_t(k) * n + i) * 128 + c] = out[k];
  if (c == 0)
    rho[i] = rsum;
}

constexpr int kTile = 8; // edges per shared-memory reduction round

template <int L, bool Accumulate>
__global__ void __launch_bounds__(128) message_backward_proj_kernel(
    int n, int r0, int e_base, const int *row, const int *sender, const float4 *vec, const float *R,
    const float *dR, const float *Y, const float *dY, const float2 *cut, const float2 *den, const float *up,
    const float *Wb, TPValues cg, const float *msg_grad, const float *rho_grad, float *up_grad,
    float4 *edge_force) {
  using T = Traits<L>;
  constexpr int P = T::P, NC = T::NC, IN = T::IN;
  __shared__ float red[2][4][kTile][4];
  int i = r0 + blockIdx.x, c = threadIdx.x, lane = c & 31, warp = c >> 5;
  float G[NC];
#pragma unroll
  for (int k = 0; k < NC; ++k)
    G[k] = msg_grad[(size_t(k) * n + i) * 128 + c];
  float bias[P];
#pragma unroll
  for (int p = 0; p < P; ++p)
    bias[p] = Wb[p * 128 + c];
  float rg = rho_grad[i];
  int begin = row[i], end = row[i + 1];
  for (int base = begin, tile = 0; base < end; base += kTile, ++tile) {
    int cnt = min(kTile, end - base);
    float(*rd)[kTile][4] = red[tile & 1];
#pragma unroll 1
    for (int k = 0; k < cnt; ++k) {
      int e = base + k;
      size_t off = size_t(e - e_base) * (P * 128) + c;
      float rv[P], drv[P];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        rv[p] = __ldcs(R + off + p * 128);
        drv[p] = __ldcs(dR + off + p * 128);
      }
      int j = __ldg(sender + e);
      float2 cv = __ldg(cut + e);
      float u[IN];
#pragma unroll
      for (int q = 0; q < IN; ++q)
        u[q] = __ldg(up + (size_t(q) * n + j) * 128 + c);
      float y[16];
      const float4 *y4 = reinterpret_cast<const float4 *>(Y + size_t(e) * 16);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float4 v = __ldg(y4 + q);
        y[4 * q] = v.x, y[4 * q + 1] = v.y, y[4 * q + 2] = v.z, y[4 * q + 3] = v.w;
      }
      float w[P], dw[P];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        float s = rv[p] + bias[p];
        w[p] = cv.x * s;
        dw[p] = cv.x * drv[p] + cv.y * s;
      }
      float Q[P], Tsh[16], ug[IN];
#pragma unroll
      for (int p = 0; p < P; ++p)
        Q[p] = 0.f;
#pragma unroll
      for (int q = 0; q < 16; ++q)
        Tsh[q] = 0.f;
#pragma unroll
      for (int q = 0; q < IN; ++q)
        ug[q] = 0.f;
      Unroll<0, T::NT>::run([&](auto tc) {
        constexpr int t = decltype(tc)::value;
        constexpr TPTerm q = T::term(t);
        float x = cg.v[t] * G[q.out];
        float xu = x * u[q.in];
        Q[q.path] = fmaf(xu, y[q.sh], Q[q.path]);
        Tsh[q.sh] = fmaf(xu, w[q.path], Tsh[q.sh]);
        if constexpr (L > 0)
          ug[q.in] = fmaf(x, y[q.sh] * w[q.path], ug[q.in]);
      });
      if constexpr (L > 0) {
#pragma unroll
        for (int q = 0; q < IN; ++q)
          atomicAdd(up_grad + (size_t(q) * n + j) * 128 + c, ug[q]);
      }
      float dr = 0.f;
#pragma unroll
      for (int p = 0; p < P; ++p)
        dr = fmaf(Q[p], dw[p], dr);
      float gx = 0.f, gy = 0.f, gz = 0.f;
      const float4 *g4 = reinterpret_cast<const float4 *>(dY + size_t(e) * 48);
#pragma unroll
      for (int q = 0; q < 12; ++q) {
        float4 v = __ldg(g4 + q);
        float gv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          int idx = 4 * q + m, sh = idx / 3, ax = idx % 3;
          float &g = ax == 0 ? gx : ax == 1 ? gy : gz;
          g = fmaf(Tsh[sh], gv[m], g);
        }
      }
      dr = warp_allsum(dr);
      gx = warp_allsum(gx);
      gy = warp_allsum(gy);
      gz = warp_allsum(gz);
      if (lane == 0) {
        rd[warp][k][0] = dr;
        rd[warp][k][1] = gx;
        rd[warp][k][2] = gy;
        rd[warp][k][3] = gz;
      }
    }
    __syncthreads();
    if (c < cnt) {
      int e = base + c;
      float s[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        s[q] = rd[0][c][q] + rd[1][c][q] + rd[2][c][q] + rd[3][c][q];
      float4 v = vec[e];
      float r = v.w > 0.f ? v.w : 1e-10f;
      float drt = s[0] + rg * den[e].y;
      float4 f = make_float4(s[1] + drt * v.x / r, s[2] + drt * v.y / r, s[3] + drt * v.z / r, 0.f);
      if (Accumulate) {
        float4 o = edge_force[e];
        f.x += o.x, f.y += o.y, f.z += o.z;
      }
      edge_force[e] = f;
    }
  }
}
} // namespace

void launch_message_forward_proj(cudaStream_t s, int layer, const DeviceGeometry &g, const Layer &l, EdgeArrays ea,
                                 RadialOut ro, const ProjectionChunk &k, const float *R, const float *up,
                                 float *message, float *density) {
  int blocks = k.r1 - k.r0;
  if (blocks <= 0)
    return;
  if (layer == 0)
    lapis::launch(message_forward_proj_kernel<0>, blocks, 128, 0, s, g.n, k.r0, int(k.e0), g.edge_offsets,
                  g.edge_sender, R, ea.Y, ea.cut, ro.density, up, l.radial.out_b, l.tp, message, density);
  else
    lapis::launch(message_forward_proj_kernel<1>, blocks, 128, 0, s, g.n, k.r0, int(k.e0), g.edge_offsets,
                  g.edge_sender, R, ea.Y, ea.cut, ro.density, up, l.radial.out_b, l.tp, message, density);
}

void launch_message_backward_proj(cudaStream_t s, int layer, const DeviceGeometry &g, const Layer &l,
                                  EdgeArrays ea, RadialOut ro, const ProjectionChunk &k, const float *R,
                                  const float *dR, const float *up, const float *message_grad,
                                  const float *density_grad, float *up_grad, float4 *edge_force, bool accumulate) {
  int blocks = k.r1 - k.r0;
  if (blocks <= 0)
    return;
#define MH1_BWD(L, A)                                                                                              \
  lapis::launch(message_backward_proj_kernel<L, A>, blocks, 128, 0, s, g.n, k.r0, int(k.e0), g.edge_offsets,       \
                g.edge_sender, g.edge_vector, R, dR, ea.Y, ea.dY, ea.cut, ro.density, up, l.radial.out_b, l.tp,     \
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
} // namespace mace
