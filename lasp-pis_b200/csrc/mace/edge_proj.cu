// Edge tensor-product kernels over a precomputed radial projection.
//
// The radial projection of the reference's MH1Pair (mace/src/mh1.cu:331-353) times the
// envelope, w[e][p*128 + c] = cut_e (sum_a h[e][a] W[a][p*128 + c] + b[p*128 + c]), and its
// r-derivative dw = cut dR + dcut (R + b), come from dense E x 64 x (P*128) GEMMs per layer
// over rows the radial kernel has already scaled:
//     R' = (cut h) W,   dR' = (cut dh + dcut h) W,   then  w = R' + cut b,  dw = dR' + dcut b.
// They run on the tensor cores (tc_gemm, fp16 hi/lo split with FP32 drains) into an HBM
// buffer, chunked by receivers, and the kernels below consume them:
//   forward   messages and density, as mace/src/mh1.cu:331-389;
//   backward  tensor-product adjoints, r-tangent and per-edge force, as mh1.cu:390-452.
// The backward regroups the term sum into per-path Q_p = sum_t cg G[out] u[in] Y[sh] (then
// dE/dr = sum_p Q_p dw_p), per-harmonic T_sh = sum_t cg G[out] u[in] w_p (then
// dE/dd = sum_sh T_sh dY_sh) and the sender up-gradient sum_t cg G[out] Y[sh] w_p, and
// factors u[in] and w_p out of each (path, in) group of terms: three FP32 operations per term
// plus three per group.  dY comes precomputed from the geometry kernel.
//
// CTA per receiver: warps 0..3 are the channels (thread = channel), warp 4 streams the
// receiver's edges through a 2- to 4-stage shared-memory ring in tiles of T edges with bulk
// copies completing on an mbarrier -- the R (and dR) rows (contiguous, receiver-major),
// the sender's up-projected features, Y (and dY) -- plus per-edge metadata, so the channel
// warps read only shared memory.  Per-edge scalars are reduced over the 128 channels with
// warp shuffles and a 4-warp shared-memory sum in a fixed order.  Waits are bounded.
#include "../lapis/launch.cuh"
#include "edge_common.cuh"
#include "model.hpp"
#include "tcgen05.cuh"
#include <cuda_fp16.h>
#include <type_traits>

namespace mace {
using lapis::DeviceGeometry;
namespace {
using namespace edge;
using tc::bulk_load;
using tc::mbar_arrive;
using tc::mbar_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::smem_u32;

constexpr int kStatusEdgeTimeout = 8;

// Channel values: a thread owns one channel (float) or two adjacent channels (float2, whose
// arithmetic runs as paired FP32 instructions, fma.rn.f32x2 / mul.rn.f32x2).
__device__ __forceinline__ float vfma(float a, float b, float c) { return fmaf(a, b, c); }
__device__ __forceinline__ float2 vfma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float vmul(float a, float b) { return a * b; }
__device__ __forceinline__ float2 vmul(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float hsum(float a) { return a; }
__device__ __forceinline__ float hsum(float2 a) { return a.x + a.y; }
template <class V> __device__ __forceinline__ V bcast(float x);
template <> __device__ __forceinline__ float bcast<float>(float x) { return x; }
template <> __device__ __forceinline__ float2 bcast<float2>(float x) { return make_float2(x, x); }
template <class V> __device__ __forceinline__ V vzero() { return bcast<V>(0.f); }

// Channel pairing per instantiation: the layer-1 backward keeps one channel per thread (its
// register budget for two channels would leave one warp per scheduler).
template <int L, bool Bwd> struct Lanes {
  static constexpr bool kPair = !(L == 1 && Bwd);
  static constexpr int W = kPair ? 2 : 1;        // channels per thread
  static constexpr int kChanThreads = 128 / W;    // channel threads per CTA
  static constexpr int kChanWarps = kChanThreads / 32;
  static constexpr int kThreads = kChanThreads + 32; // plus the producer warp
  static constexpr int kMinBlocks = L ? (Bwd ? 3 : 4) : (Bwd ? 5 : 8);
  using V = std::conditional_t<kPair, float2, float>;
};

struct EdgeMeta {
  float4 vec; // d, r
  float2 cut, den;
  int sender, row, pad[2]; // row: e - e_base (the edge's row in the chunk buffers)
};

template <int L, bool Bwd> struct Stage {
  static constexpr int P = Traits<L>::P, IN = Traits<L>::IN;
  // Edges per tile: layer 0 (16 terms per edge) takes 4 so that the per-tile channel reduction
  // and its barrier are paid less often per edge.
  static constexpr int T = L ? 2 : 4;
  // Ring depth: the layer-1 backward keeps 2 stages (50 KB) so that 3 CTAs fit an SM at its
  // 128 registers, the layer-1 forward 3 (44 KB, 4 CTAs); layer 0 keeps 8 edges in flight.
  static constexpr int NS = L ? (Bwd ? 2 : 3) : 2;
  static constexpr int ROW = P * 128 * 4;             // bytes of one R row
  static constexpr int R = 0, DR = R + T * ROW, U = DR + (Bwd ? T * ROW : 0), Y = U + T * IN * 512;
  static constexpr int DY = Y + T * 64, META = DY + (Bwd ? T * 192 : 0), EF = META + T * sizeof(EdgeMeta);
  // EF: an accumulating backward's current per-edge forces, copied in with the tile.
  // UG: the layer-1 backward's per-edge up-gradient rows, written by the channel threads and
  // copied out to global memory in one bulk store per tile.
  static constexpr int UG = EF + (Bwd ? T * 16 : 0);
  static constexpr int BYTES = UG + (Bwd && L > 0 ? T * IN * 512 : 0);
  static constexpr unsigned tx(int cnt, bool forces) {
    return cnt * ((Bwd ? 2 : 1) * ROW + IN * 512 + 64 + (Bwd ? 192 : 0) + (forces ? 16 : 0));
  }
};

struct ProjArgs {
  int n, r0, e_base;
  int n_up; // row stride of up / up_grad (the sender count)
  const int *row, *sender;
  const float4 *vec;
  const float *R, *dR, *Y, *dY; // R', dR' (see above)
  const float2 *cut, *den;
  const float *up, *bias;
  const float *msg_grad, *rho_grad; // backward inputs
  float *msg, *rho;                 // forward outputs
  SplitPlanes msg_split;            // forward: msg as the tensor-core linear_1's split operand
  float *ug_edge;                   // backward, layer 1: per-edge up-gradient rows [e - e_base][IN][128]
  float4 *edge_force;               // backward output
  int *status;
};

// Terms sharing (path, in) form a group; the backward factors u[in] and w[path] out of each
// group.  The tables list every group contiguously (checked below).
template <int L> constexpr bool same_group(int s, int t) {
  return Traits<L>::term(s).path == Traits<L>::term(t).path && Traits<L>::term(s).in == Traits<L>::term(t).in;
}
template <int L> constexpr bool group_start(int t) { return t == 0 || !same_group<L>(t - 1, t); }
template <int L> constexpr bool group_end(int t) { return t == Traits<L>::NT - 1 || !same_group<L>(t, t + 1); }
template <int L> constexpr bool groups_contiguous() {
  for (int s = 0; s < Traits<L>::NT; ++s)
    for (int t = s + 1; t < Traits<L>::NT; ++t)
      if (same_group<L>(s, t) && !same_group<L>(t - 1, t))
        return false;
  return true;
}
static_assert(groups_contiguous<0>() && groups_contiguous<1>(), "tensor-product groups must be contiguous");

// Sums of (v0, v1, v2, v3) over the warp: lane 0 gets v0, lane 2 v1, lane 1 v2, lane 3 v3
// (component 2 * (lane & 1) + ((lane >> 1) & 1)).  Halving exchanges, then a butterfly:
// 6 shuffles instead of 20.
__device__ __forceinline__ float warp_sum4(float v0, float v1, float v2, float v3, int lane) {
  bool b0 = lane & 1, b1 = lane & 2;
  float k0 = b0 ? v2 : v0, k1 = b0 ? v3 : v1;
  k0 += __shfl_xor_sync(0xffffffffu, b0 ? v0 : v2, 1);
  k1 += __shfl_xor_sync(0xffffffffu, b0 ? v1 : v3, 1);
  float k = b1 ? k1 : k0;
  k += __shfl_xor_sync(0xffffffffu, b1 ? k0 : k1, 2);
  k += __shfl_xor_sync(0xffffffffu, k, 4);
  k += __shfl_xor_sync(0xffffffffu, k, 8);
  k += __shfl_xor_sync(0xffffffffu, k, 16);
  return k;
}

// OR of `x` over the `count` channel threads (named barrier 1); also a barrier among them.
__device__ __forceinline__ bool channels_any(bool x, int count) {
  unsigned r;
  asm volatile("{\n\t.reg .pred p, q;\n\t"
               "setp.ne.u32 q, %1, 0;\n\t"
               "bar.red.or.pred p, 1, %2, q;\n\t"
               "selp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(r)
               : "r"(unsigned(x)), "r"(count)
               : "memory");
  return r != 0;
}

template <int L, bool Bwd, bool Accumulate>
__global__ void __launch_bounds__(Lanes<L, Bwd>::kThreads, Lanes<L, Bwd>::kMinBlocks)
    edge_proj_kernel(ProjArgs a, TPValues cg) {
  using S = Stage<L, Bwd>;
  using Tr = Traits<L>;
  using LN = Lanes<L, Bwd>;
  using V = typename LN::V;
  constexpr int P = Tr::P, NC = Tr::NC, IN = Tr::IN, T = S::T, kStages = S::NS;
  constexpr int W = LN::W, kCW = LN::kChanWarps, kCT = LN::kChanThreads;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t bars[2 * kStages]; // full[s] | empty[s]
  __shared__ float red[2][kCW][T][4];
  __shared__ volatile int abort_flag;
  int i = a.r0 + blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int begin = a.row[i], end = a.row[i + 1], ntiles = (end - begin + T - 1) / T;
  unsigned full0 = smem_u32(bars), empty0 = full0 + 8 * kStages;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full0 + 8 * s, 32);
      mbar_init(empty0 + 8 * s, kCT);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // Bulk store of tile t's up-gradient rows (layer-1 backward): rows e0 - e_base .. of the
  // chunk buffer are contiguous (consecutive edges).  Producer lane 0 only.
  auto store_ug_rows = [&](int t, unsigned char *st) {
    int e0 = begin + t * T, cnt = min(T, end - e0);
    tc::bulk_store(a.ug_edge + size_t(e0 - a.e_base) * IN * 128, smem_u32(st + S::UG), unsigned(cnt) * IN * 512);
    tc::bulk_commit();
  };
  (void)store_ug_rows;

  if (warp == kCW) {
    // ---------------- producer ----------------
    // The forward reads edge metadata 32 edges (32 / T tiles) at a time, one edge per lane, so
    // the global round trip is paid once per chunk; the backward, whose tiles take longer,
    // reads it per tile.
    constexpr int kChunkTiles = Bwd ? 1 : 32 / T;
    bool run = true;
    for (int c0 = 0; c0 < ntiles && run; c0 += kChunkTiles) {
      int me = begin + c0 * T + lane, j = 0;
      EdgeMeta m{};
      if (lane < kChunkTiles * T && me < end) {
        m.vec = a.vec[me];
        m.cut = a.cut[me];
        m.den = a.den[me];
        m.sender = j = a.sender[me];
        m.row = me - a.e_base;
      }
      int tend = min(ntiles, c0 + kChunkTiles);
      for (int t = c0; t < tend; ++t) {
        int s = t % kStages;
        bool ok = t < kStages || mbar_wait(empty0 + 8 * s, ((t / kStages) - 1) & 1, &abort_flag);
        if (!__all_sync(0xffffffffu, ok)) {
          run = false;
          break;
        }
        unsigned char *st = smem + s * S::BYTES;
        unsigned sb = smem_u32(st), full = full0 + 8 * s;
        if constexpr (Bwd && L > 0) {
          // Tile t - NS, consumed (its up-gradient rows written and fenced): store its rows,
          // and let the store finish reading the stage before the stage is refilled.
          if (t >= kStages && lane == 0) {
            store_ug_rows(t - kStages, st);
            tc::bulk_wait_read();
          }
        }
        int e0 = begin + t * T, cnt = min(T, end - e0), k = lane - (t - c0) * T;
        bool mine = k >= 0 && k < cnt; // this lane holds the tile's edge k
        if (mine)
          reinterpret_cast<EdgeMeta *>(st + S::META)[k] = m;
        __syncwarp();
        if (lane == 0)
          mbar_expect_tx(full, S::tx(cnt, Bwd && Accumulate));
        __syncwarp();
        if (lane == 0) {
          size_t r = size_t(e0 - a.e_base) * (P * 128);
          bulk_load(sb + S::R, a.R + r, cnt * S::ROW, full);
          if constexpr (Bwd)
            bulk_load(sb + S::DR, a.dR + r, cnt * S::ROW, full);
          bulk_load(sb + S::Y, a.Y + size_t(e0) * 16, cnt * 64, full);
          if constexpr (Bwd)
            bulk_load(sb + S::DY, a.dY + size_t(e0) * 48, cnt * 192, full);
          if constexpr (Bwd && Accumulate)
            bulk_load(sb + S::EF, a.edge_force + e0, cnt * 16, full);
        }
        if (mine) {
#pragma unroll
          for (int q = 0; q < IN; ++q)
            bulk_load(sb + S::U + (k * IN + q) * 512, a.up + (size_t(q) * a.n_up + j) * 128, 512, full);
        }
        if (lane != 0)
          mbar_arrive(full);
      }
    }
    if constexpr (Bwd && L > 0) {
      // The last NS tiles' rows, once the channel warps are done with them.
      for (int t = max(0, ntiles - kStages); t < ntiles && run; ++t) {
        int s = t % kStages;
        bool ok = mbar_wait(empty0 + 8 * s, (t / kStages) & 1, &abort_flag);
        if (!__all_sync(0xffffffffu, ok))
          break;
        if (lane == 0)
          store_ug_rows(t, smem + s * S::BYTES);
      }
      if (lane == 0)
        tc::bulk_wait(); // complete before the CTA's shared memory is released
    }
    return;
  }

  // ---------------- channels ----------------
  // Thread c owns channels W c .. W c + W - 1; V holds them.
  int c = threadIdx.x;
  constexpr int CS = 128 / W; // stride of one 128-channel row in V units
  V bias[P];
#pragma unroll
  for (int p = 0; p < P; ++p)
    bias[p] = reinterpret_cast<const V *>(a.bias)[p * CS + c];
  V acc[Bwd ? 1 : NC], G[Bwd ? NC : 1];
  float rg = 0.f, rsum = 0.f;
  if constexpr (Bwd) {
#pragma unroll
    for (int k = 0; k < NC; ++k)
      G[k] = reinterpret_cast<const V *>(a.msg_grad)[(size_t(k) * a.n + i) * CS + c];
    rg = a.rho_grad[i];
  } else {
#pragma unroll
    for (int k = 0; k < NC; ++k)
      acc[k] = vzero<V>();
  }
  bool ok = true;
  for (int t = 0; t < ntiles; ++t) {
    int s = t % kStages;
    ok = mbar_wait(full0 + 8 * s, (t / kStages) & 1, &abort_flag);
    if (channels_any(!ok, kCT)) {
      ok = false;
      break;
    }
    const unsigned char *st = smem + s * S::BYTES;
    const EdgeMeta *meta = reinterpret_cast<const EdgeMeta *>(st + S::META);
    int cnt = min(T, end - (begin + t * T));
    if constexpr (Bwd && L > 0) {
      // This thread's entries of the stage's up-gradient rows start at zero (the bulk store
      // that last read them finished before the barrier above).
      float *ugs = reinterpret_cast<float *>(const_cast<unsigned char *>(st) + S::UG) + c;
#pragma unroll
      for (int q = 0; q < T * IN; ++q)
        ugs[q * 128] = 0.f;
    }
    for (int k = 0; k < cnt; ++k) {
      const V *Rk = reinterpret_cast<const V *>(st + S::R + k * S::ROW) + c;
      const V *Uk = reinterpret_cast<const V *>(st + S::U + k * IN * 512) + c;
      const float4 *Y4 = reinterpret_cast<const float4 *>(st + S::Y + k * 64);
      float2 cv = meta[k].cut;
      V u[IN];
      float y[16];
#pragma unroll
      for (int q = 0; q < IN; ++q)
        u[q] = Uk[q * CS];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float4 v = Y4[q];
        y[4 * q] = v.x, y[4 * q + 1] = v.y, y[4 * q + 2] = v.z, y[4 * q + 3] = v.w;
      }
      if constexpr (!Bwd) {
        V w[P];
#pragma unroll
        for (int p = 0; p < P; ++p)
          w[p] = vfma(bcast<V>(cv.x), bias[p], Rk[p * CS]);
        V uw = vzero<V>();
        Unroll<0, Tr::NT>::run([&](auto tc_) {
          constexpr int tt = decltype(tc_)::value;
          constexpr TPTerm q = Tr::term(tt);
          if constexpr (group_start<L>(tt))
            uw = vmul(u[q.in], w[q.path]);
          acc[q.out] = vfma(bcast<V>(cg.v[tt] * y[q.sh]), uw, acc[q.out]);
        });
        rsum += meta[k].den.x;
      } else {
        const V *dRk = reinterpret_cast<const V *>(st + S::DR + k * S::ROW) + c;
        // dw = dcut b + dR' is formed after the term loop, where it is used (fewer live registers).
        V w[P];
#pragma unroll
        for (int p = 0; p < P; ++p)
          w[p] = vfma(bcast<V>(cv.x), bias[p], Rk[p * CS]);
        V Q[P], Tsh[16], ug[IN];
#pragma unroll
        for (int p = 0; p < P; ++p)
          Q[p] = vzero<V>();
#pragma unroll
        for (int q = 0; q < 16; ++q)
          Tsh[q] = vzero<V>();
#pragma unroll
        for (int q = 0; q < IN; ++q)
          ug[q] = vzero<V>();
        // Per group (p, in) with a_t = cg_t G[out_t] and S = sum_t a_t Y[sh_t]:
        //   Q_p += u[in] S,   ug[in] += w_p S,   T_sh += a_t (u[in] w_p)
        // -- three operations per term plus three per group.
        V S = vzero<V>(), uw = vzero<V>();
        Unroll<0, Tr::NT>::run([&](auto tc_) {
          constexpr int tt = decltype(tc_)::value;
          constexpr TPTerm q = Tr::term(tt);
          V at = vmul(bcast<V>(cg.v[tt]), G[q.out]);
          if constexpr (group_start<L>(tt)) {
            uw = vmul(u[q.in], w[q.path]);
            S = vmul(at, bcast<V>(y[q.sh]));
          } else {
            S = vfma(at, bcast<V>(y[q.sh]), S);
          }
          Tsh[q.sh] = vfma(at, uw, Tsh[q.sh]);
          if constexpr (group_end<L>(tt)) {
            Q[q.path] = vfma(u[q.in], S, Q[q.path]);
            if constexpr (L > 0)
              ug[q.in] = vfma(w[q.path], S, ug[q.in]);
          }
        });
        if constexpr (L > 0) {
          // An add onto the zeroed slot (0 + x = x exactly): a reduction instruction here keeps
          // the compiler from interleaving the next edge's loads, which would spill registers.
          static_assert(W == 1, "the up-gradient staging assumes one channel per thread");
          float *dst = reinterpret_cast<float *>(const_cast<unsigned char *>(st) + S::UG + k * IN * 512) + c;
#pragma unroll
          for (int q = 0; q < IN; ++q)
            atomicAdd(dst + q * 128, hsum(ug[q]));
        }
        V dr2 = vzero<V>();
#pragma unroll
        for (int p = 0; p < P; ++p)
          dr2 = vfma(Q[p], vfma(bcast<V>(cv.y), bias[p], dRk[p * CS]), dr2);
        V g2[3] = {vzero<V>(), vzero<V>(), vzero<V>()};
        const float4 *g4 = reinterpret_cast<const float4 *>(st + S::DY + k * 192);
#pragma unroll
        for (int q = 0; q < 12; ++q) {
          float4 v = g4[q];
          float gv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            int idx = 4 * q + m, sh = idx / 3, ax = idx % 3;
            g2[ax] = vfma(Tsh[sh], bcast<V>(gv[m]), g2[ax]);
          }
        }
        float sum = warp_sum4(hsum(dr2), hsum(g2[0]), hsum(g2[1]), hsum(g2[2]), lane);
        if (lane < 4)
          red[t & 1][warp][k][2 * (lane & 1) + (lane >> 1)] = sum;
      }
    }
    if constexpr (Bwd) {
      if constexpr (L > 0)
        tc::fence_proxy_async_smem(); // the up-gradient rows, for the producer's bulk store
      asm volatile("bar.sync 1, %0;" ::"r"(kCT) : "memory");
      if (c < cnt) {
        int e = begin + t * T + c;
        float sum[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          sum[q] = red[t & 1][0][c][q];
#pragma unroll
          for (int w = 1; w < kCW; ++w)
            sum[q] += red[t & 1][w][c][q];
        }
        float4 v = meta[c].vec;
        float r = v.w > 0.f ? v.w : 1e-10f;
        float drt = sum[0] + rg * meta[c].den.y;
        float4 f = make_float4(sum[1] + drt * v.x / r, sum[2] + drt * v.y / r, sum[3] + drt * v.z / r, 0.f);
        if (Accumulate) {
          float4 o = reinterpret_cast<const float4 *>(st + S::EF)[c];
          f.x += o.x, f.y += o.y, f.z += o.z;
        }
        a.edge_force[e] = f;
      }
    }
    mbar_arrive(empty0 + 8 * s);
  }
  if constexpr (!Bwd) {
    if (ok) {
      if (a.msg_split.hi) {
        // A warp's 64 channels are one 64-wide slab of each message row: its maximum by
        // shuffles, then the fp16 hi / lo pair of each channel.
        static_assert(W == 2, "the split message write assumes two channels per thread");
#pragma unroll
        for (int k = 0; k < NC; ++k) {
          float2 v = acc[k];
          // Warp maximum as an integer reduction of |v|'s bit patterns (ordered like the values).
          float m = __uint_as_float(
              __reduce_max_sync(0xffffffffu, __float_as_uint(fmaxf(fabsf(v.x), fabsf(v.y)))));
          int e = tc::split_exponent(m);
          float sc = __uint_as_float(uint32_t(127 + e) << 23);
          float2 x = __fmul2_rn(v, make_float2(sc, sc));
          __half2 h = __float22half2_rn(x);
          __half2 l = __float22half2_rn(__ffma2_rn(__half22float2(h), make_float2(-1.f, -1.f), x));
          size_t el = (size_t(k) * a.n + i) * 128 + 2 * c;
          *reinterpret_cast<__half2 *>(a.msg_split.hi + el) = h;
          *reinterpret_cast<__half2 *>(a.msg_split.lo + el) = l;
          if (lane == 0)
            a.msg_split.exp[el / 64] = int16_t(e);
        }
      } else {
#pragma unroll
        for (int k = 0; k < NC; ++k)
          reinterpret_cast<V *>(a.msg)[(size_t(k) * a.n + i) * CS + c] = acc[k];
      }
      if (c == 0)
        a.rho[i] = rsum;
    }
  }
  if (!ok) {
    if (c == 0)
      atomicCAS(a.status, 0, kStatusEdgeTimeout);
    // Let the copies already issued land before the CTA's shared memory is released.
    if (c < kStages) {
      long long start = clock64();
      int last = ntiles - 1 - ((ntiles - 1 - c) % kStages);
      while (last >= 0 && !tc::mbar_try(full0 + 8 * (last % kStages), (last / kStages) & 1) &&
             clock64() - start < tc::kWaitCycles) {
      }
    }
  }
}

template <int L, bool Bwd, bool Accumulate>
void launch_proj(cudaStream_t s, int blocks, const ProjArgs &a, const TPValues &cg) {
  constexpr int smem = Stage<L, Bwd>::NS * Stage<L, Bwd>::BYTES;
  lapis::check(
      cudaFuncSetAttribute(edge_proj_kernel<L, Bwd, Accumulate>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  lapis::launch(edge_proj_kernel<L, Bwd, Accumulate>, blocks, Lanes<L, Bwd>::kThreads, smem, s, a, cg);
}

ProjArgs proj_args(const DeviceGeometry &g, const Layer &l, EdgeArrays ea, RadialOut ro, const ProjectionChunk &k,
                   const float *R, const float *up, int n_up) {
  ProjArgs a{};
  a.n = g.n;
  a.n_up = n_up ? n_up : g.n;
  a.r0 = k.r0;
  a.e_base = int(k.e0);
  a.row = g.edge_offsets;
  a.sender = g.edge_sender;
  a.vec = g.edge_vector;
  a.R = R;
  a.Y = ea.Y;
  a.dY = ea.dY;
  a.den = ro.density;
  a.up = up;
  a.cut = ea.cut;
  a.bias = l.radial.out_b;
  a.status = g.status;
  return a;
}
} // namespace

void launch_message_forward_proj(cudaStream_t s, int layer, const DeviceGeometry &g, const Layer &l, EdgeArrays ea,
                                 RadialOut ro, const ProjectionChunk &k, const float *R, const float *up,
                                 float *message, float *density, int n_up, SplitPlanes message_split) {
  int blocks = k.r1 - k.r0;
  if (blocks <= 0)
    return;
  ProjArgs a = proj_args(g, l, ea, ro, k, R, up, n_up);
  a.msg = message;
  a.rho = density;
  a.msg_split = message_split;
  if (layer == 0)
    launch_proj<0, false, false>(s, blocks, a, l.tp);
  else
    launch_proj<1, false, false>(s, blocks, a, l.tp);
}

void launch_message_backward_proj(cudaStream_t s, int layer, const DeviceGeometry &g, const Layer &l,
                                  EdgeArrays ea, RadialOut ro, const ProjectionChunk &k, const float *R,
                                  const float *dR, const float *up, const float *message_grad,
                                  const float *density_grad, float *ug_edge, float4 *edge_force, bool accumulate,
                                  int n_up) {
  int blocks = k.r1 - k.r0;
  if (blocks <= 0)
    return;
  ProjArgs a = proj_args(g, l, ea, ro, k, R, up, n_up);
  a.dR = dR;
  a.msg_grad = message_grad;
  a.rho_grad = density_grad;
  a.ug_edge = ug_edge;
  a.edge_force = edge_force;
  if (layer == 0) {
    if (accumulate)
      launch_proj<0, true, true>(s, blocks, a, l.tp);
    else
      launch_proj<0, true, false>(s, blocks, a, l.tp);
  } else {
    if (accumulate)
      launch_proj<1, true, true>(s, blocks, a, l.tp);
    else
      launch_proj<1, true, false>(s, blocks, a, l.tp);
  }
}
} // namespace mace
