// Lennard-Jones through the PairOp API (lapis/examples/lj/lj.cu in the reference): the
// force-shifted potential u(r) = 4 eps [(s/r)^12 - (s/r)^6] - u_c - (r - r_c) u'_c.
// Thread = edge of a 128-edge tile, per-thread accumulators, then a warp-shuffle + 4-warp
// shared-memory reduction per receiver in finalize.
#include "lapis/lj.h"
#include "lapis/lj.hpp"
#include "lapis/pair.cuh"
#include <cmath>
#include <string>

namespace lapis {
void set_c_api_error(const std::string &);
namespace {
struct LJOp {
  static constexpr int threads = 128, tile_edges = 128, scratch_alignment = 16;
  static const char *name() { return "LennardJones"; }
  struct State {
    float e, f[3], v[9];
  };
  float epsilon, sigma, rc, uc, duc;
  float *energy, *force, *virial;
  int *status;
  WorkspaceSpec plan(int) const { return {0, 4 * 13 * sizeof(float), 16}; }
  void setup(Context &, void *) {}
  void postprocess(Context &, void *) {}
  __device__ void prepare(int, State &s, void *) {
    s.e = 0.f;
    for (int k = 0; k < 3; ++k)
      s.f[k] = 0.f;
    for (int k = 0; k < 9; ++k)
      s.v[k] = 0.f;
  }
  template <class Tile> __device__ void consume(int, const Tile &tile, State &s, void *) {
    int e = threadIdx.x;
    if (e >= tile.size())
      return;
    float r2 = tile.squared_distance(e);
    if (r2 <= 0.f) {
      atomicCAS(status, 0, 1);
      return;
    }
    float r = sqrtf(r2), q = sigma * sigma / r2, q6 = q * q * q;
    float u = 4.f * epsilon * (q6 * q6 - q6) - uc - (r - rc) * duc;
    float du = 24.f * epsilon * (q6 - 2.f * q6 * q6) / r - duc;
    float3 d = tile.displacement(e);
    float x[3] = {d.x, d.y, d.z};
    s.e += .5f * u;
#pragma unroll
    for (int k = 0; k < 3; ++k)
      s.f[k] += du * x[k] / r;
#pragma unroll
    for (int k = 0; k < 3; ++k)
#pragma unroll
      for (int l = 0; l < 3; ++l)
        s.v[3 * k + l] -= .5f * du * x[k] * x[l] / r;
  }
  __device__ void finalize(int i, State &s, void *scratch) {
    float *red = static_cast<float *>(scratch); // [4 warps][13]
    float acc[13] = {s.e, s.f[0], s.f[1], s.f[2], s.v[0], s.v[1], s.v[2], s.v[3], s.v[4], s.v[5], s.v[6], s.v[7], s.v[8]};
    int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int k = 0; k < 13; ++k) {
#pragma unroll
      for (int o = 16; o; o >>= 1)
        acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], o);
      if (lane == 0)
        red[warp * 13 + k] = acc[k];
    }
    __syncthreads();
    if (threadIdx.x < 13) {
      int k = threadIdx.x;
      float v = red[k] + red[13 + k] + red[26 + k] + red[39 + k];
      if (k == 0)
        energy[i] = v;
      else if (k < 4)
        force[3 * i + k - 1] = v;
      else
        virial[9 * i + k - 4] = v;
    }
  }
};
} // namespace

LennardJones::LennardJones(float e, float s, float c, Options o) : Calculator(c, o), epsilon_(e), sigma_(s) {
  if (!std::isfinite(e) || e <= 0 || !std::isfinite(s) || s <= 0 || !std::isfinite(c) || c <= 0)
    throw Error("Invalid LJ parameters");
}

Result LennardJones::evaluate() {
  int n = context_.geometry.n;
  float *e = context_.array<float>("lj.e", n), *f = context_.array<float>("lj.f", 3 * size_t(n)),
        *v = context_.array<float>("lj.v", 9 * size_t(n));
  float a = std::pow(sigma_ / cutoff_, 6.f), uc = 4 * epsilon_ * (a * a - a),
        duc = 24 * epsilon_ * (a - 2 * a * a) / cutoff_;
  execute(context_, LJOp{epsilon_, sigma_, cutoff_, uc, duc, e, f, v, context_.geometry.status});
  return context_.finish(e, f, v);
}
} // namespace lapis

extern "C" int lapis_lj_calculate(int n, const float *xyz, const int *Z, const float *cell, float epsilon,
                                  float sigma, float cutoff, int backend, double *energy, float *per_atom,
                                  float *force, float *virial) {
  try {
    if (n < 0 || !cell || !energy || (n > 0 && (!xyz || !Z || !per_atom || !force)) || !virial)
      throw lapis::Error("Invalid LJ arguments");
    if (backend < 0 || backend > 2)
      throw lapis::Error("Invalid neighbor backend");
    lapis::Options o;
    o.backend = lapis::NeighborBackend(backend);
    lapis::LennardJones lj(epsilon, sigma, cutoff, o);
    lapis::Structure s;
    s.size = n;
    s.positions = xyz;
    s.elements = Z;
    for (int k = 0; k < 9; ++k)
      s.cell[k] = cell[k];
    auto r = lj.calculate(s);
    *energy = r.energy;
    for (int i = 0; i < n; ++i)
      per_atom[i] = r.energies[i];
    for (int k = 0; k < 3 * n; ++k)
      force[k] = r.forces[k];
    for (int k = 0; k < 9; ++k)
      virial[k] = r.virial[k];
    return 0;
  } catch (const std::exception &e) {
    lapis::set_c_api_error(e.what());
    return -1;
  }
}
