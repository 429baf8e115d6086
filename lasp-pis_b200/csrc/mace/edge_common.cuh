// Device math shared by the SIMT and tensor-core edge kernels: forward-mode tangents,
// envelope, component-normalised real harmonics with gradients, the compiled per-layer
// tensor-product traits and a compile-time unroller.  Mathematics as in the reference's
// mace/src/mh1_math.cuh (D1, envelope, harmonics) and mace/src/mh1.cu:297-316.
#pragma once
#include "model.hpp"
#include <type_traits>

namespace mace {
namespace edge {
// ---------------- small forward-mode tangents (value, d/dr) ----------------
struct D1 {
  float v, d;
};
__device__ __forceinline__ D1 operator+(D1 a, D1 b) { return {a.v + b.v, a.d + b.d}; }
__device__ __forceinline__ D1 operator-(D1 a, D1 b) { return {a.v - b.v, a.d - b.d}; }
__device__ __forceinline__ D1 operator*(D1 a, D1 b) { return {a.v * b.v, a.d * b.v + a.v * b.d}; }
__device__ __forceinline__ D1 operator/(D1 a, D1 b) {
  float v = a.v / b.v;
  return {v, (a.d - v * b.d) / b.v};
}
__device__ __forceinline__ D1 cst(float x) { return {x, 0.f}; }
__device__ __forceinline__ D1 dpow(D1 a, float b) {
  float v = powf(a.v, b);
  return {v, b * v / a.v * a.d};
}
__device__ __forceinline__ D1 dexp(D1 a) {
  float v = expf(a.v);
  return {v, v * a.d};
}
__device__ __forceinline__ D1 dsin(D1 a) { return {sinf(a.v), cosf(a.v) * a.d}; }
__device__ __forceinline__ D1 envelope(D1 r, float rc, float p) {
  if (r.v >= rc)
    return {0.f, 0.f};
  D1 x = r / cst(rc);
  return cst(1.f) - cst((p + 1) * (p + 2) * .5f) * dpow(x, p) + cst(p * (p + 2)) * dpow(x, p + 1) -
         cst(p * (p + 1) * .5f) * dpow(x, p + 2);
}
// Logistic sigmoid; __frcp_rn is the correctly rounded reciprocal, i.e. the same value as the
// IEEE division 1 / y.
__device__ __forceinline__ float sigm(float x) { return __frcp_rn(1.f + expf(-x)); }

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int s = 16; s; s >>= 1)
    v += __shfl_xor_sync(0xffffffffu, v, s);
  return v;
}

// Component-normalised harmonics of u = -d/r; optionally dY/dd (G[k][b]).
template <bool Grad> __device__ __forceinline__ void harmonics(float dx, float dy, float dz, float r, float *Y,
                                                             float (*G)[3]) {
  float ir = 1.f / r;
  float x = -dx * ir, y = -dy * ir, z = -dz * ir;
  const float s3 = 1.7320508075688772f, s5 = 2.23606797749979f, a9 = .9128709291752769f,
              a11 = .6123724356957945f;
  float yy = y * y, xxzz = x * x + z * z;
  float s4 = s3 * x * z, s8 = .8660254037844386f * (z * z - x * x);
  float P[16];
  P[0] = 1.f;
  P[1] = x;
  P[2] = y;
  P[3] = z;
  P[4] = s4;
  P[5] = s3 * x * y;
  P[6] = yy - .5f * xxzz;
  P[7] = s3 * y * z;
  P[8] = s8;
  P[9] = a9 * (s4 * z + s8 * x);
  P[10] = s5 * s4 * y;
  float t = 4.f * yy - xxzz;
  P[11] = a11 * t * x;
  float t2 = 2.f * yy - 3.f * xxzz;
  P[12] = .5f * y * t2;
  P[13] = a11 * z * t;
  P[14] = s5 * s8 * y;
  P[15] = a9 * (s8 * z - s4 * x);
  const float norm[4] = {1.f, 1.7320508075688772f, 2.23606797749979f, 2.6457513110645907f};
#pragma unroll
  for (int k = 0; k < 16; ++k)
    Y[k] = P[k] * norm[k == 0 ? 0 : k < 4 ? 1 : k < 9 ? 2 : 3];
  if constexpr (Grad) {
    float D[16][3];
    float g4[3] = {s3 * z, 0.f, s3 * x}, g8[3] = {-s3 * x, 0.f, s3 * z};
    float dt[3] = {-2.f * x, 8.f * y, -2.f * z}, dt2[3] = {-6.f * x, 4.f * y, -6.f * z};
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      float ex = q == 0, ey = q == 1, ez = q == 2;
      D[0][q] = 0.f;
      D[1][q] = ex;
      D[2][q] = ey;
      D[3][q] = ez;
      D[4][q] = g4[q];
      D[5][q] = s3 * (ex * y + x * ey);
      D[6][q] = 2.f * y * ey - x * ex - z * ez;
      D[7][q] = s3 * (ey * z + y * ez);
      D[8][q] = g8[q];
      D[9][q] = a9 * (g4[q] * z + s4 * ez + g8[q] * x + s8 * ex);
      D[10][q] = s5 * (g4[q] * y + s4 * ey);
      D[11][q] = a11 * (dt[q] * x + t * ex);
      D[12][q] = .5f * (t2 * ey + y * dt2[q]);
      D[13][q] = a11 * (t * ez + z * dt[q]);
      D[14][q] = s5 * (g8[q] * y + s8 * ey);
      D[15][q] = a9 * (g8[q] * z + s8 * ez - g4[q] * x - s4 * ex);
    }
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      float s = norm[k == 0 ? 0 : k < 4 ? 1 : k < 9 ? 2 : 3];
      float du = D[k][0] * x + D[k][1] * y + D[k][2] * z;
      G[k][0] = -s * ir * (D[k][0] - du * x);
      G[k][1] = -s * ir * (D[k][1] - du * y);
      G[k][2] = -s * ir * (D[k][2] - du * z);
    }
  }
}

// ---------------- per-layer compile-time traits ----------------
template <int L> struct Traits;
template <> struct Traits<0> {
  static constexpr int P = 4, NC = 16, IN = 1, NT = kTPTerms0, EC = 8;
  static constexpr TPTerm term(int t) { return kTP0[t]; }
};
template <> struct Traits<1> {
  static constexpr int P = 10, NC = 40, IN = 4, NT = kTPTerms1, EC = 4;
  static constexpr TPTerm term(int t) { return kTP1[t]; }
};

template <int I, int N> struct Unroll {
  template <class F> __device__ __forceinline__ static void run(F &&f) {
    f(std::integral_constant<int, I>{});
    Unroll<I + 1, N>::run(f);
  }
};
template <int N> struct Unroll<N, N> {
  template <class F> __device__ __forceinline__ static void run(F &&) {}
};

} // namespace edge
} // namespace mace
