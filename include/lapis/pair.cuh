// Lapis L1 PairOp extension API (drop-in for lapis/include/lapis/pair.cuh and the contract in
// lapis/docs/PAIR_OP.md of the reference): `lapis::execute(context, op)` runs a user
// operation over every receiver's directed periodic edges.
//
// An operation is a trivially device-copyable value with
//   static constexpr int threads (multiple of 32, <= 1024), tile_edges (> 0),
//                        scratch_alignment (power of two in [16, 256]);
//   optional static constexpr int edge_threads (divides threads) and static dim3 block_shape();
//   static const char *name();  struct State;
//   WorkspaceSpec plan(int atoms) const;  void setup(Context&, void*);  void postprocess(Context&, void*);
//   __device__ void prepare(int receiver, State&, void *scratch);
//   template <class Tile> __device__ void consume(int receiver, const Tile&, State&, void *scratch);
//   __device__ void finalize(int receiver, State&, void *scratch);
//
// B200 build: the edges already exist as the CSR list that Context::prepare enumerated once
// (full directed edges including periodic self-images, excluding (i, i, 0), inclusive
// cutoff), so one CTA per receiver streams its consecutive CSR edges through two alternating
// shared-memory SoA tiles of `tile_edges` edges -- one barrier per tile -- and every thread
// calls prepare, consume (once per tile, the last tile partial) and finalize in the same
// order.  TileView accessors are shared-memory loads; squared_distance is the float32 value
// the traversal compared against the cutoff.  Sender/receiver ids are internal
// (spatially sorted) node ids; Context holds the maps to the caller's order.
#pragma once
#include "runtime.hpp"
#include <climits>
#include <string>
#include <type_traits>

namespace lapis {
// Flattened CTA rank of the calling thread (for operations with a multidimensional block).
__device__ inline int thread_rank() {
  return threadIdx.x + blockDim.x * (threadIdx.y + blockDim.y * threadIdx.z);
}

namespace pair_detail {
template <class Op, class = void> struct BlockShape {
  static constexpr bool flat = true;
  static dim3 get() { return dim3(Op::threads, 1, 1); }
};
template <class Op> struct BlockShape<Op, std::void_t<decltype(Op::block_shape())>> {
  static constexpr bool flat = false;
  static dim3 get() { return Op::block_shape(); }
};
template <class Op, class = void> struct EdgeThreads {
  static constexpr int value = 1;
};
template <class Op> struct EdgeThreads<Op, std::void_t<decltype(Op::edge_threads)>> {
  static constexpr int value = Op::edge_threads;
};
__host__ __device__ constexpr size_t round_up(size_t n, size_t a) { return (n + a - 1) & ~(a - 1); }

// One tile of edges, structure of arrays.
template <int T> struct alignas(16) EdgeTile {
  int sender[T], sx[T], sy[T], sz[T];
  float dx[T], dy[T], dz[T], r2[T];
};
} // namespace pair_detail

template <int T> struct TileView {
  const pair_detail::EdgeTile<T> *tile;
  int count;
  __device__ int size() const { return count; }
  __device__ int sender(int e) const { return tile->sender[e]; }
  __device__ int3 shift(int e) const { return make_int3(tile->sx[e], tile->sy[e], tile->sz[e]); }
  __device__ float3 displacement(int e) const { return make_float3(tile->dx[e], tile->dy[e], tile->dz[e]); }
  __device__ float squared_distance(int e) const { return tile->r2[e]; }
};

template <class Op> __global__ void pair_kernel(DeviceGeometry g, Op op) {
  constexpr int T = Op::tile_edges;
  using Tile = pair_detail::EdgeTile<T>;
  extern __shared__ __align__(256) unsigned char pair_storage[];
  Tile *tiles = reinterpret_cast<Tile *>(pair_storage);
  void *scratch = pair_storage + pair_detail::round_up(2 * sizeof(Tile), Op::scratch_alignment);
  int t = pair_detail::BlockShape<Op>::flat ? int(threadIdx.x) : thread_rank(), i = blockIdx.x;
  typename Op::State state{};
  op.prepare(i, state, scratch);
  int begin = g.edge_offsets[i], end = g.edge_offsets[i + 1];
  for (int base = begin, k = 0; base < end; base += T, ++k) {
    // Tile k goes to buffer k & 1: every thread finished consuming tile k - 2 (which used
    // that buffer) before the barrier of tile k - 1.
    Tile &tile = tiles[k & 1];
    int count = min(T, end - base);
    for (int e = t; e < count; e += Op::threads) {
      int edge = base + e;
      float4 v = g.edge_vector[edge];
      tile.sender[e] = g.edge_sender[edge];
      tile.sx[e] = g.edge_shift[3 * edge];
      tile.sy[e] = g.edge_shift[3 * edge + 1];
      tile.sz[e] = g.edge_shift[3 * edge + 2];
      tile.dx[e] = v.x;
      tile.dy[e] = v.y;
      tile.dz[e] = v.z;
      tile.r2[e] = g.edge_r2[edge];
    }
    __syncthreads();
    op.consume(i, TileView<T>{&tile, count}, state, scratch);
  }
  op.finalize(i, state, scratch);
}

// Checks the operation against the device, records its resources, reserves its workspace,
// then setup -> traversal kernel on ctx.stream -> postprocess (lapis/include/lapis/pair.cuh:
// 179-225 in the reference, same checks and messages).
template <class Op> void execute(Context &ctx, Op op) {
  static_assert(Op::threads > 0 && Op::threads % 32 == 0 && Op::threads <= 1024, "PairOp thread count");
  static_assert(Op::tile_edges > 0, "PairOp tile size");
  static_assert(Op::scratch_alignment >= 16 && Op::scratch_alignment <= 256 &&
                    (Op::scratch_alignment & (Op::scratch_alignment - 1)) == 0,
                "PairOp scratch alignment");
  static_assert(pair_detail::EdgeThreads<Op>::value > 0 && Op::threads % pair_detail::EdgeThreads<Op>::value == 0,
                "PairOp edge subgroup");
  WorkspaceSpec plan = op.plan(ctx.geometry.n);
  if (plan.scratch_alignment != size_t(Op::scratch_alignment))
    throw Error("PairOp scratch alignment mismatch");
  dim3 block = pair_detail::BlockShape<Op>::get();
  if (size_t(block.x) * block.y * block.z != size_t(Op::threads))
    throw Error("PairOp block shape does not match thread count");
  if (plan.scratch_bytes > 1024 * 1024)
    throw Error("PairOp dynamic scratch exceeds supported per-block storage");
  size_t shared = pair_detail::round_up(2 * sizeof(pair_detail::EdgeTile<Op::tile_edges>), Op::scratch_alignment) +
                  plan.scratch_bytes;
  cudaFuncAttributes attr{};
  check(cudaFuncGetAttributes(&attr, pair_kernel<Op>));
  int device = 0;
  check(cudaGetDevice(&device));
  cudaDeviceProp props{};
  check(cudaGetDeviceProperties(&props, device));
  if (block.x > unsigned(props.maxThreadsDim[0]) || block.y > unsigned(props.maxThreadsDim[1]) ||
      block.z > unsigned(props.maxThreadsDim[2]))
    throw Error("PairOp block dimension exceeds device limit");
  if (Op::threads > attr.maxThreadsPerBlock || shared + attr.sharedSizeBytes > props.sharedMemPerBlockOptin ||
      size_t(attr.numRegs) * Op::threads > size_t(props.regsPerBlock))
    throw Error("PairOp exceeds device kernel resource limits");
  if (shared + attr.sharedSizeBytes > props.sharedMemPerBlock)
    check(cudaFuncSetAttribute(pair_kernel<Op>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(shared)));
  int active = 0;
  check(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&active, pair_kernel<Op>, Op::threads, shared));
  if (active < 1)
    throw Error("PairOp has no resident block capacity");
  ctx.resources.push_back({Op::name(), attr.numRegs, Op::threads, active, attr.sharedSizeBytes, shared});
  void *workspace = ctx.reserve(std::string("op.") + Op::name(), plan.global_bytes);
  op.setup(ctx, workspace);
  if (ctx.geometry.n) {
    ++launch_counter();
    pair_kernel<Op><<<ctx.geometry.n, block, shared, ctx.stream>>>(ctx.geometry, op);
  }
  check(cudaGetLastError());
  op.postprocess(ctx, workspace);
}
} // namespace lapis
