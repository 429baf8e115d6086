// Deterministic sender-side sums over the receiver-major CSR edge list.
//
// Two quantities of the MH1 backward flow from an edge to its SENDER: the layer-1
// up-projection gradient (512 floats per edge) and, in a domain-decomposed evaluation, the
// reaction force on a ghost sender.  The reference scatters both with global float atomics
// (mace/src/mh1.cu:411-413), so its forces change in the last bits from call to call.  This
// build writes each edge's contribution once and then sums it on the sender's side
// ("owner computes"): a sender index lists, per sender, its edges in ascending edge order,
// and a gather kernel adds them in that order.  The sums are therefore the same on every
// call, on every handle and for every chunking of the edge list.
//
// Sender index (built once per evaluation): count per sender, exclusive scan, placement with
// an atomic cursor (arbitrary order), then each sender's segment sorted by edge id, which
// makes the final order independent of the placement.
#include "../lapis/launch.cuh"
#include "model.hpp"

namespace mace {
namespace {
__global__ void count_senders(long long E, const int *sender, int *counts) {
  long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (e < E)
    atomicAdd(counts + sender[e], 1);
}

// Exclusive scan of n ints by one CTA of 1024 threads; out[n] = total.
__global__ void scan_counts(const int *in, int *out, int n) {
  __shared__ int partial[1024];
  int t = threadIdx.x;
  int chunk = (n + 1023) / 1024, begin = min(n, t * chunk), end = min(n, begin + chunk), s = 0;
  for (int k = begin; k < end; ++k)
    s += in[k];
  partial[t] = s;
  __syncthreads();
  for (int step = 1; step < 1024; step *= 2) {
    int v = t >= step ? partial[t - step] : 0;
    __syncthreads();
    partial[t] += v;
    __syncthreads();
  }
  int run = t ? partial[t - 1] : 0;
  for (int k = begin; k < end; ++k) {
    out[k] = run;
    run += in[k];
  }
  if (t == 1023)
    out[n] = partial[1023];
}

__global__ void place_edges(long long E, const int *sender, const int *offsets, int *cursor, int *slots) {
  long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (e < E) {
    int j = sender[e];
    slots[offsets[j] + atomicAdd(cursor + j, 1)] = int(e);
  }
}

// Warp per sender: every entry of the segment goes to position (number of smaller entries);
// entries are distinct edge ids.  Segments up to kSortStage entries are staged in shared
// memory, longer ones are ranked from global memory.
constexpr int kSortThreads = 256, kSortStage = 256;
__global__ void __launch_bounds__(kSortThreads) sort_segments(int n, const int *offsets, const int *slots,
                                                              int *sorted) {
  __shared__ int stage[kSortThreads / 32][kSortStage];
  int j = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (j >= n)
    return;
  int begin = offsets[j], len = offsets[j + 1] - begin;
  const int *seg = slots + begin;
  if (len <= kSortStage) {
    int *v = stage[threadIdx.x >> 5];
    for (int k = lane; k < len; k += 32)
      v[k] = seg[k];
    __syncwarp();
    seg = v;
  }
  for (int k = lane; k < len; k += 32) {
    int x = seg[k], rank = 0;
    for (int q = 0; q < len; ++q)
      rank += seg[q] < x;
    sorted[begin + rank] = x;
  }
}

// First position in list[b, e) with list[k] >= key (the list is ascending).
__device__ __forceinline__ int lower_bound(const int *list, int b, int e, long long key) {
  while (b < e) {
    int m = (b + e) >> 1;
    if (list[m] < key)
      b = m + 1;
    else
      e = m;
  }
  return b;
}

// Warp per sender j: out[q][j][c] += sum over j's edges e in [e0, e1), ascending, of
// rows[e - e0][q][c] (C components of 128 channels; a lane owns 4 channels as a float4).
template <int C>
__global__ void sender_gather_kernel(int n, const int *offsets, const int *list, long long e0, long long e1,
                                     const float *rows, float *out, int stride) {
  int j = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (j >= n)
    return;
  int b = lower_bound(list, offsets[j], offsets[j + 1], e0), end = offsets[j + 1];
  if (b >= end || list[b] >= e1)
    return;
  float4 acc[C];
#pragma unroll
  for (int q = 0; q < C; ++q)
    acc[q] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = b; k < end; ++k) {
    long long e = list[k];
    if (e >= e1)
      break;
    const float4 *r = reinterpret_cast<const float4 *>(rows + size_t(e - e0) * C * 128) + lane;
#pragma unroll
    for (int q = 0; q < C; ++q) {
      float4 v = __ldcs(r + q * 32);
      acc[q].x += v.x, acc[q].y += v.y, acc[q].z += v.z, acc[q].w += v.w;
    }
  }
#pragma unroll
  for (int q = 0; q < C; ++q) {
    float4 *o = reinterpret_cast<float4 *>(out + (size_t(q) * stride + j) * 128) + lane;
    float4 v = *o;
    v.x += acc[q].x, v.y += acc[q].y, v.z += acc[q].z, v.w += acc[q].w;
    *o = v;
  }
}

// Warp per ghost sender j in [n_own, n_local): force[j] -= sum of its edges' forces (lanes
// take edges in a fixed stride, then a fixed butterfly sum).
__global__ void ghost_reaction_kernel(int n_own, int n_local, const int *offsets, const int *list, const float4 *ef,
                                      float *force) {
  int j = n_own + ((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (j >= n_local)
    return;
  float sx = 0.f, sy = 0.f, sz = 0.f;
  for (int k = offsets[j] + lane; k < offsets[j + 1]; k += 32) {
    float4 f = ef[list[k]];
    sx += f.x, sy += f.y, sz += f.z;
  }
  for (int m = 16; m; m >>= 1) {
    sx += __shfl_xor_sync(0xffffffffu, sx, m);
    sy += __shfl_xor_sync(0xffffffffu, sy, m);
    sz += __shfl_xor_sync(0xffffffffu, sz, m);
  }
  if (lane == 0) {
    force[3 * j] -= sx;
    force[3 * j + 1] -= sy;
    force[3 * j + 2] -= sz;
  }
}

inline int grid_for(long long threads, int block) { return int(std::max<long long>(1, (threads + block - 1) / block)); }
} // namespace

SenderIndex build_sender_index(cudaStream_t s, lapis::Context &c, long long E, int n_senders, const int *sender) {
  SenderIndex si{n_senders, c.array<int>("mh.sender.offsets", size_t(n_senders) + 1),
                 c.array<int>("mh.sender.edges", size_t(std::max<long long>(E, 1)))};
  int *counts = c.array<int>("mh.sender.counts", size_t(n_senders) + 1);
  int *slots = c.array<int>("mh.sender.slots", size_t(std::max<long long>(E, 1)));
  c.clear(counts, (size_t(n_senders) + 1) * sizeof(int));
  if (E)
    lapis::launch(count_senders, grid_for(E, 256), 256, 0, s, E, sender, counts);
  lapis::launch(scan_counts, 1, 1024, 0, s, counts, si.offsets, n_senders);
  if (E) {
    c.clear(counts, size_t(n_senders) * sizeof(int)); // reused as the placement cursor
    lapis::launch(place_edges, grid_for(E, 256), 256, 0, s, E, sender, si.offsets, counts, slots);
    lapis::launch(sort_segments, grid_for(size_t(n_senders) * 32, kSortThreads), kSortThreads, 0, s, n_senders,
                  si.offsets, slots, si.edges);
  }
  return si;
}

void launch_sender_gather(cudaStream_t s, const SenderIndex &si, long long e0, long long e1, const float *rows,
                          int comps, float *out, int stride) {
  if (e1 <= e0 || !si.n)
    return;
  if (comps != 4)
    throw lapis::Error("sender gather: unsupported component count");
  lapis::launch(sender_gather_kernel<4>, grid_for(size_t(si.n) * 32, 256), 256, 0, s, si.n, si.offsets, si.edges, e0,
                e1, rows, out, stride);
}

void launch_ghost_reactions(cudaStream_t s, const SenderIndex &si, int n_own, const float4 *edge_force,
                            float *force) {
  if (si.n > n_own)
    lapis::launch(ghost_reaction_kernel, grid_for(size_t(si.n - n_own) * 32, 256), 256, 0, s, n_own, si.n,
                  si.offsets, si.edges, edge_force, force);
}
} // namespace mace
