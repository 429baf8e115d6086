// Tensor-core (tcgen05) edge kernels: the per-edge radial projection 64 -> P x 128 of the
// reference's MH1Pair (mace/src/mh1.cu:331-353) runs as a UMMA with the channels on the
// TMEM lanes, fused with the channel-wise tensor product that consumes it
// (mace/src/mh1.cu:370-389) and, for the backward, with the tensor-product adjoints, the
// r-tangent and the per-edge force (mace/src/mh1.cu:390-452).
//
// One persistent CTA per SM owns a contiguous range of receivers and walks their CSR
// edges in tiles of ET edges.  For every tile and path p:
//     D_p[c][e] = sum_a W9[p*128 + c][a] * h[e][a]          (M = 128 channels, K = 64)
// with the weights split at load into tf32 hi + lo and the edge features split on the fly,
// accumulated in TMEM as W_hi*h_hi + W_lo*h_hi + W_hi*h_lo.  The backward stacks the
// tangent dh/dr of the same edges as extra MMA columns (N = 2 x ET), so w and its
// r-derivative come out of the same instructions.
//
// Warps: 0 TMA producer (edge features per tile, the P x 2 weight slabs through a
// 3-stage ring), 1 MMA issuer, 2..5 epilogue (lane = channel; tensor product or adjoints
// from TMEM, messages accumulated per receiver in registers -- a receiver never spans two
// CTAs, so no atomics), 6..7 split the edge features into tf32 hi/lo.  Waits are bounded.
#include "../lapis/launch.cuh"
#include "edge_common.cuh"
#include "model.hpp"
#include "tcgen05.cuh"
#include <cuda.h>

namespace mace {
namespace {
using namespace tc;
using namespace edge;
using lapis::DeviceGeometry;

constexpr int kStatusEdgeTimeout = 8;
constexpr int kWStages = 3, kWSlab = 128 * 32 * 4; // one path x 32-wide K slab, 16 KiB
constexpr int kThreads = 256;

template <int L, bool Bwd> struct Shape {
  static constexpr int P = Traits<L>::P, NC = Traits<L>::NC, IN = Traits<L>::IN, NT_ = Traits<L>::NT;
  static constexpr int N = L == 0 ? 96 : 48;        // MMA N (columns per path)
  static constexpr int ET = Bwd ? N / 2 : N;        // edges per tile
  static constexpr int COLS = P * N;                // TMEM columns used
  static constexpr int ALLOC = COLS <= 256 ? 256 : 512;
  static constexpr int BREG = N * 128;              // bytes of one 32-wide K slab of B rows
  static constexpr int BBUF = 4 * BREG;             // hi kh0 | hi kh1 | lo kh0 | lo kh1
  static constexpr int G = Bwd ? 4 : 8;             // edges per TMEM load group
  static constexpr uint32_t IDESC = idesc_tf32(128, N);
};

// Byte offsets of the per-tile metadata that follows the operand buffers.
template <int L, bool Bwd> struct Meta {
  static constexpr int ET = Shape<L, Bwd>::ET;
  static constexpr int ys = 0, gys = ys + ET * 64, cut = gys + (Bwd ? ET * 192 : 0), den = cut + ET * 8;
  static constexpr int vec = (den + ET * 4 + 15) / 16 * 16, snd = vec + ET * 16, rg = snd + ET * 4;
  static constexpr int red = rg + ET * 4, bar = (red + 64 * ET + 7) / 8 * 8, bytes = bar + 16 * 8;
};

struct EdgeTCArgs {
  int n;
  const int *row, *sender;
  const float4 *vec;
  const float *Y;
  const float2 *cut, *den;
  const float *up, *bias;
  const float *msg_grad, *rho_grad; // backward inputs
  float *msg, *rho;                 // forward outputs
  float *up_grad;                   // backward (layer 1)
  float4 *edge_force;               // backward output
  int accumulate_force;
  int receivers_per_cta;
  int *status;
};

// OR of `x` over the 128 epilogue threads (named barrier 1); also a barrier among them.
__device__ __forceinline__ bool epilogue_any(bool x) {
  unsigned r;
  asm volatile("{\n\t.reg .pred p, q;\n\t"
               "setp.ne.u32 q, %1, 0;\n\t"
               "bar.red.or.pred p, 1, 128, q;\n\t"
               "selp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(r)
               : "r"(unsigned(x))
               : "memory");
  return r != 0;
}

template <int L, bool Bwd>
__global__ void __launch_bounds__(kThreads, 1)
    edge_tc_kernel(const __grid_constant__ CUtensorMap tmH, const __grid_constant__ CUtensorMap tmDH,
                   const __grid_constant__ CUtensorMap tmWhi, const __grid_constant__ CUtensorMap tmWlo,
                   EdgeTCArgs a, TPValues cg) {
  using S = Shape<L, Bwd>;
  using T = Traits<L>;
  constexpr int P = S::P, NC = S::NC, IN = S::IN, N = S::N, ET = S::ET, G = S::G;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using M = Meta<L, Bwd>;
  unsigned char *wring = smem;                        // kWStages x (hi | lo)
  unsigned char *bbuf = smem + kWStages * 2 * kWSlab; // 2 x BBUF
  unsigned char *meta = bbuf + 2 * S::BBUF;
  float *ys = reinterpret_cast<float *>(meta + M::ys);    // [ET][16]
  float *gys = reinterpret_cast<float *>(meta + M::gys);  // [ET][16][3] (backward)
  float2 *cuts = reinterpret_cast<float2 *>(meta + M::cut);
  float *dens = reinterpret_cast<float *>(meta + M::den); // den value (fwd) / d den/dr (bwd)
  float4 *vecs = reinterpret_cast<float4 *>(meta + M::vec);
  int *snds = reinterpret_cast<int *>(meta + M::snd);
  float *rgs = reinterpret_cast<float *>(meta + M::rg);   // receiver density grad per edge
  float *red = reinterpret_cast<float *>(meta + M::red);  // [4 warps][ET][4]
  uint64_t *bars = reinterpret_cast<uint64_t *>(meta + M::bar);
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ int final_issued;
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // barriers: wfull[3] wempty[3] bfull[2] bready[2] bempty[2] accfull accempty
  unsigned wfull0 = smem_u32(bars), wempty0 = wfull0 + 8 * kWStages, bfull0 = wempty0 + 8 * kWStages,
           bready0 = bfull0 + 16, bempty0 = bready0 + 16, accfull = bempty0 + 16, accempty = accfull + 8;
  int r0 = blockIdx.x * a.receivers_per_cta, r1 = min(a.n, r0 + a.receivers_per_cta);
  if (r0 >= r1)
    return;
  int e_begin = a.row[r0], e_end = a.row[r1];
  int ntiles = (e_end - e_begin + ET - 1) / ET;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    final_issued = 0;
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(wfull0 + 8 * s, 1);
      mbar_init(wempty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bfull0 + 8 * b, 1);
      mbar_init(bready0 + 8 * b, 64);
      mbar_init(bempty0 + 8 * b, 1);
    }
    mbar_init(accfull, 1);
    mbar_init(accempty, 128);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(S::ALLOC));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int ws = 0;
      for (int t = 0; t < ntiles; ++t) {
        int buf = t & 1, e0 = e_begin + t * ET;
        if (t >= 2 && !mbar_wait(bempty0 + 8 * buf, ((t >> 1) - 1) & 1, &abort_flag))
          break;
        unsigned b = smem_u32(bbuf + buf * S::BBUF);
        mbar_expect_tx(bfull0 + 8 * buf, 2 * S::BREG);
        for (int kh = 0; kh < 2; ++kh) {
          tma_load_2d(b + kh * S::BREG, &tmH, 32 * kh, e0, bfull0 + 8 * buf);
          if constexpr (Bwd)
            tma_load_2d(b + kh * S::BREG + ET * 128, &tmDH, 32 * kh, e0, bfull0 + 8 * buf);
        }
        bool ok = true;
        for (int p = 0; p < P && ok; ++p)
          for (int kh = 0; kh < 2; ++kh, ++ws) {
            int st = ws % kWStages;
            if (ws >= kWStages && !(ok = mbar_wait(wempty0 + 8 * st, ((ws / kWStages) - 1) & 1, &abort_flag)))
              break;
            unsigned w = smem_u32(wring + st * 2 * kWSlab);
            mbar_expect_tx(wfull0 + 8 * st, 2 * kWSlab);
            tma_load_2d(w, &tmWhi, 32 * kh, 128 * p, wfull0 + 8 * st);
            tma_load_2d(w + kWSlab, &tmWlo, 32 * kh, 128 * p, wfull0 + 8 * st);
          }
        if (!ok)
          break;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int ws = 0;
      bool ok = true;
      for (int t = 0; t < ntiles && ok; ++t) {
        int buf = t & 1;
        ok = mbar_wait(bready0 + 8 * buf, (t >> 1) & 1, &abort_flag);
        if (ok && t >= 1)
          ok = mbar_wait(accempty, (t - 1) & 1, &abort_flag);
        if (!ok)
          break;
        tc_fence_after();
        unsigned b = smem_u32(bbuf + buf * S::BBUF);
        for (int p = 0; p < P && ok; ++p)
          for (int kh = 0; kh < 2; ++kh, ++ws) {
            int st = ws % kWStages;
            if (!(ok = mbar_wait(wfull0 + 8 * st, (ws / kWStages) & 1, &abort_flag)))
              break;
            tc_fence_after();
            unsigned w = smem_u32(wring + st * 2 * kWSlab);
            uint32_t d = tmem + uint32_t(p * N);
            // The tensor pipe truncates each accumulation toward zero, with an error relative
            // to the accumulator: the small correction terms go first (K half 0: while the
            // accumulator is small) and the dominant hi*hi terms after them.
            if (kh == 0) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                uint64_t whi = smem_desc(w + 32 * j), wlo = smem_desc(w + kWSlab + 32 * j);
                uint64_t bhi = smem_desc(b + 32 * j), blo = smem_desc(b + 2 * S::BREG + 32 * j);
                umma_tf32_desc(d, wlo, bhi, S::IDESC, j ? 1u : 0u);
                umma_tf32_desc(d, whi, blo, S::IDESC, 1u);
                umma_tf32_desc(d, whi, bhi, S::IDESC, 1u);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                uint64_t whi = smem_desc(w + 32 * j), wlo = smem_desc(w + kWSlab + 32 * j);
                uint64_t bhi = smem_desc(b + S::BREG + 32 * j), blo = smem_desc(b + 3 * S::BREG + 32 * j);
                umma_tf32_desc(d, wlo, bhi, S::IDESC, 1u);
                umma_tf32_desc(d, whi, blo, S::IDESC, 1u);
              }
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                uint64_t whi = smem_desc(w + 32 * j);
                uint64_t bhi = smem_desc(b + S::BREG + 32 * j);
                umma_tf32_desc(d, whi, bhi, S::IDESC, 1u);
              }
            }
            umma_commit(wempty0 + 8 * st);
          }
        if (!ok)
          break;
        umma_commit(bempty0 + 8 * buf);
        umma_commit(accfull);
      }
      final_issued = 1;
    }
  } else if (warp >= 6) {
    // ---------------- edge-feature split (hi / lo) ----------------
    int tid = threadIdx.x - 192;
    for (int t = 0; t < ntiles; ++t) {
      int buf = t & 1;
      bool ok = mbar_wait(bfull0 + 8 * buf, (t >> 1) & 1, &abort_flag);
      if (!__all_sync(0xffffffffu, ok))
        break;
      float4 *hi = reinterpret_cast<float4 *>(bbuf + buf * S::BBUF);
      float4 *lo = reinterpret_cast<float4 *>(bbuf + buf * S::BBUF + 2 * S::BREG);
      for (int q = tid; q < 2 * S::BREG / 16; q += 64) {
        float4 v = hi[q], h, l;
        h.x = tf32_hi(v.x), h.y = tf32_hi(v.y), h.z = tf32_hi(v.z), h.w = tf32_hi(v.w);
        l.x = v.x - h.x, l.y = v.y - h.y, l.z = v.z - h.z, l.w = v.w - h.w;
        hi[q] = h;
        lo[q] = l;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(bready0 + 8 * buf);
    }
  } else {
    // ---------------- epilogue: lane = channel ----------------
    int quarter = warp & 3, c = 32 * quarter + lane, te = threadIdx.x - 64;
    uint32_t lane_addr = tmem + (uint32_t(32 * quarter) << 16);
    float bias[P];
#pragma unroll
    for (int p = 0; p < P; ++p)
      bias[p] = a.bias[p * 128 + c];
    int ri = r0, seg_end = a.row[r0 + 1];
    float acc[NC], G_[NC], rsum = 0.f, rg = 0.f;
#pragma unroll
    for (int k = 0; k < NC; ++k)
      acc[k] = 0.f, G_[k] = 0.f;
    auto enter = [&](int r) {
      if constexpr (Bwd) {
#pragma unroll
        for (int k = 0; k < NC; ++k)
          G_[k] = a.msg_grad[(size_t(k) * a.n + r) * 128 + c];
        rg = a.rho_grad[r];
      }
    };
    auto flush = [&]() {
      if constexpr (!Bwd) {
#pragma unroll
        for (int k = 0; k < NC; ++k) {
          a.msg[(size_t(k) * a.n + ri) * 128 + c] = acc[k];
          acc[k] = 0.f;
        }
        if (c == 0)
          a.rho[ri] = rsum;
        rsum = 0.f;
      }
    };
    enter(ri);
    bool ok = true;
    for (int t = 0; t < ntiles && ok; ++t) {
      int e0 = e_begin + t * ET, cnt = min(ET, e_end - e0);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      for (int idx = te; idx < cnt * 16; idx += 128)
        ys[idx] = a.Y[size_t(e0) * 16 + idx];
      if (te < cnt) {
        int e = e0 + te;
        cuts[te] = a.cut[e];
        snds[te] = a.sender[e];
        float2 dn = a.den[e];
        dens[te] = Bwd ? dn.y : dn.x;
        if constexpr (Bwd) {
          float4 v = a.vec[e];
          float r = v.w > 0.f ? v.w : 1e-10f;
          vecs[te] = make_float4(v.x, v.y, v.z, r);
          float Yv[16], Gv[16][3];
          harmonics<true>(v.x, v.y, v.z, r, Yv, Gv);
          for (int k = 0; k < 16; ++k)
            for (int q = 0; q < 3; ++q)
              gys[(te * 16 + k) * 3 + q] = Gv[k][q];
        }
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      ok = mbar_wait(accfull, t & 1, &abort_flag);
      // All 128 epilogue threads take the same decision (they share named barrier 1).
      if (epilogue_any(!ok)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int g0 = 0; g0 < cnt; g0 += G) {
        float w[P][G], dw[Bwd ? P : 1][G];
#pragma unroll
        for (int p = 0; p < P; ++p) {
            if constexpr (!Bwd) {
            tmem_ld8(lane_addr + uint32_t(p * N + g0), w[p]);
          } else {
            // w for edges g0..g0+3 and their tangent projections at column offset ET
            tmem_ld4(lane_addr + uint32_t(p * N + g0), w[p]);
            tmem_ld4(lane_addr + uint32_t(p * N + ET + g0), dw[p]);
          }
        }
        tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < G; ++q) {
          int el = g0 + q;
          if (el >= cnt)
            break;
          int e = e0 + el;
          while (e >= seg_end) {
            flush();
            ++ri;
            seg_end = a.row[ri + 1];
            enter(ri);
          }
          int j = snds[el];
          float u[IN];
#pragma unroll
          for (int k = 0; k < IN; ++k)
            u[k] = a.up[(size_t(k) * a.n + j) * 128 + c];
          float2 cv = cuts[el];
          const float *ye = ys + el * 16;
          if constexpr (!Bwd) {
            float wp[P];
#pragma unroll
            for (int p = 0; p < P; ++p)
              wp[p] = cv.x * (w[p][q] + bias[p]);
            Unroll<0, T::NT>::run([&](auto tc_) {
              constexpr int tt = decltype(tc_)::value;
              constexpr TPTerm qq = T::term(tt);
              acc[qq.out] = fmaf(cg.v[tt] * ye[qq.sh], u[qq.in] * wp[qq.path], acc[qq.out]);
            });
            if (c == 0)
              rsum += dens[el];
          } else {
            float wp[P], dwp[P], ug[IN];
#pragma unroll
            for (int p = 0; p < P; ++p) {
              float sv = w[p][q] + bias[p];
              wp[p] = cv.x * sv;
              dwp[p] = cv.x * dw[p][q] + cv.y * sv;
            }
#pragma unroll
            for (int k = 0; k < IN; ++k)
              ug[k] = 0.f;
            float dr = 0.f, gx = 0.f, gy = 0.f, gz = 0.f;
            const float *ge = gys + el * 48;
            Unroll<0, T::NT>::run([&](auto tc_) {
              constexpr int tt = decltype(tc_)::value;
              constexpr TPTerm qq = T::term(tt);
              float av = G_[qq.out] * cg.v[tt];
              float xv = av * u[qq.in];
              float yv = ye[qq.sh];
              dr = fmaf(xv * yv, dwp[qq.path], dr);
              float z = xv * wp[qq.path];
              gx = fmaf(z, ge[qq.sh * 3], gx);
              gy = fmaf(z, ge[qq.sh * 3 + 1], gy);
              gz = fmaf(z, ge[qq.sh * 3 + 2], gz);
              if constexpr (L > 0)
                ug[qq.in] = fmaf(av * yv, wp[qq.path], ug[qq.in]);
            });
            if constexpr (L > 0) {
#pragma unroll
              for (int k = 0; k < IN; ++k)
                atomicAdd(a.up_grad + (size_t(k) * a.n + j) * 128 + c, ug[k]);
            }
            dr = warp_allsum(dr);
            gx = warp_allsum(gx);
            gy = warp_allsum(gy);
            gz = warp_allsum(gz);
            if (lane == 0) {
              float *rd = red + (quarter * ET + el) * 4;
              rd[0] = dr, rd[1] = gx, rd[2] = gy, rd[3] = gz;
            }
            if (c == 0)
              rgs[el] = rg;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(accempty);
      if constexpr (Bwd) {
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (te < cnt) {
          float s4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            s4[q] = red[(0 * ET + te) * 4 + q] + red[(1 * ET + te) * 4 + q] + red[(2 * ET + te) * 4 + q] +
                    red[(3 * ET + te) * 4 + q];
          float4 v = vecs[te];
          float drt = s4[0] + rgs[te] * dens[te];
          float4 f = make_float4(s4[1] + drt * v.x / v.w, s4[2] + drt * v.y / v.w, s4[3] + drt * v.z / v.w, 0.f);
          if (a.accumulate_force) {
            float4 o = a.edge_force[e0 + te];
            f.x += o.x, f.y += o.y, f.z += o.z;
          }
          a.edge_force[e0 + te] = f;
        }
      }
    }
    if (ok) {
      // Close the open receiver and any trailing receivers without edges.
      while (ri < r1) {
        flush();
        ++ri;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (abort_flag && threadIdx.x == 0)
    atomicCAS(a.status, 0, kStatusEdgeTimeout);
  if (warp == 1) {
    if (abort_flag && final_issued) {
      long long start = clock64();
      while (!mbar_try(accfull, (ntiles - 1) & 1) && clock64() - start < kWaitCycles) {
      }
    }
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::ALLOC));
  }
}

// Shared memory for a specialisation (alignment slack included).
template <int L, bool Bwd> constexpr int smem_bytes() {
  return 1024 + kWStages * 2 * kWSlab + 2 * Shape<L, Bwd>::BBUF + Meta<L, Bwd>::bytes;
}
} // namespace


template <int L, bool Bwd>
void launch_edge_tc_impl(cudaStream_t s, const DeviceGeometry &g, const Layer &l, EdgeArrays ea, RadialOut ro,
                         EdgeTCArgs args) {
  using S = Shape<L, Bwd>;
  long long E = g.edge_capacity;
  CUtensorMap mh = tc_map_2d(ro.h, 64, E, 32, S::ET);
  CUtensorMap mdh = tc_map_2d(Bwd ? ro.dh : ro.h, 64, E, 32, S::ET);
  CUtensorMap whi = tc_map_2d(l.radial.out_hi, 64, (long long)S::P * 128, 32, 128);
  CUtensorMap wlo = tc_map_2d(l.radial.out_lo, 64, (long long)S::P * 128, 32, 128);
  int device = 0, sms = 148;
  lapis::check(cudaGetDevice(&device));
  lapis::check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  constexpr int smem = smem_bytes<L, Bwd>();
  lapis::check(cudaFuncSetAttribute(edge_tc_kernel<L, Bwd>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  int grid = std::min(g.n, sms);
  args.receivers_per_cta = (g.n + grid - 1) / grid;
  grid = (g.n + args.receivers_per_cta - 1) / args.receivers_per_cta;
  (void)ea;
  lapis::launch(edge_tc_kernel<L, Bwd>, grid, kThreads, smem, s, mh, mdh, whi, wlo, args, l.tp);
}

void launch_message_forward_tc(cudaStream_t s, int layer, const DeviceGeometry &g, const Layer &l, EdgeArrays ea,
                               RadialOut ro, const float *up, float *message, float *density) {
  if (!g.n)
    return;
  if (!g.edge_capacity) {
    lapis::check(cudaMemsetAsync(message, 0, size_t(g.n) * 128 * l.out_comp * 4, s));
    lapis::check(cudaMemsetAsync(density, 0, size_t(g.n) * 4, s));
    return;
  }
  EdgeTCArgs a{};
  a.n = g.n;
  a.row = g.edge_offsets;
  a.sender = g.edge_sender;
  a.vec = g.edge_vector;
  a.Y = ea.Y;
  a.cut = ea.cut;
  a.den = ro.density;
  a.up = up;
  a.bias = l.radial.out_b;
  a.msg = message;
  a.rho = density;
  a.status = g.status;
  if (layer == 0)
    launch_edge_tc_impl<0, false>(s, g, l, ea, ro, a);
  else
    launch_edge_tc_impl<1, false>(s, g, l, ea, ro, a);
}

void launch_message_backward_tc(cudaStream_t s, int layer, const DeviceGeometry &g, const Layer &l, EdgeArrays ea,
                                RadialOut ro, const float *up, const float *message_grad, const float *density_grad,
                                float *up_grad, float4 *edge_force, bool accumulate) {
  if (!g.n || !g.edge_capacity)
    return;
  EdgeTCArgs a{};
  a.n = g.n;
  a.row = g.edge_offsets;
  a.sender = g.edge_sender;
  a.vec = g.edge_vector;
  a.Y = ea.Y;
  a.cut = ea.cut;
  a.den = ro.density;
  a.up = up;
  a.bias = l.radial.out_b;
  a.msg_grad = message_grad;
  a.rho_grad = density_grad;
  a.up_grad = up_grad;
  a.edge_force = edge_force;
  a.accumulate_force = accumulate;
  a.status = g.status;
  if (layer == 0)
    launch_edge_tc_impl<0, true>(s, g, l, ea, ro, a);
  else
    launch_edge_tc_impl<1, true>(s, g, l, ea, ro, a);
}
} // namespace mace
