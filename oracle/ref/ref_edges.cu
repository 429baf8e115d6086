// TEST INFRASTRUCTURE ONLY: dumps the reference Lapis traversal's directed edges.
// Compiled against the reference's own lapis/include/lapis/pair.cuh and
// lapis/src/runtime.cu by oracle/ref/Makefile; the PairOp below is this project's code.
// It records (original receiver, original sender, shift) per tile edge, like the
// reference's edge-multiset tests do (lapis/tests/framework.cu:18-70).
#include "lapis/pair.cuh"
#include <algorithm>
#include <array>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>
using namespace lapis;
namespace {
struct Dump {
  static constexpr int threads = 128, tile_edges = 32, scratch_alignment = 16;
  static const char *name() { return "oracle.dump_edges"; }
  struct State {};
  int *edges, *count;
  int capacity;
  const int *map;
  WorkspaceSpec plan(int) const { return {0, 0, 16}; }
  void setup(Context &c, void *) { c.clear(count, 4); }
  void postprocess(Context &, void *) {}
  __device__ void prepare(int, State &, void *) {}
  template <class T> __device__ void consume(int i, const T &tile, State &, void *) {
    int t = threadIdx.x;
    if (t < tile.size()) {
      int k = atomicAdd(count, 1);
      if (k < capacity) {
        int3 s = tile.shift(t);
        edges[5 * k] = map[i];
        edges[5 * k + 1] = map[tile.sender(t)];
        edges[5 * k + 2] = s.x;
        edges[5 * k + 3] = s.y;
        edges[5 * k + 4] = s.z;
      }
    }
  }
  __device__ void finalize(int, State &, void *) {}
};
thread_local std::string last_error;
} // namespace
extern "C" __attribute__((visibility("default"))) const char *ref_edges_error() { return last_error.c_str(); }
// Returns the number of edges (sorted canonically into out[5*cap]) or -1 on error.
extern "C" __attribute__((visibility("default"))) int64_t ref_edges(int n, const float *xyz, const int *z,
                                                                    const float *cell, int backend,
                                                                    float cutoff, int64_t grid_bytes,
                                                                    int64_t cap, int *out) {
  try {
    Structure s;
    s.size = n;
    s.positions = xyz;
    s.elements = z;
    std::copy(cell, cell + 9, s.cell.begin());
    Options o;
    o.backend = NeighborBackend(backend);
    if (grid_bytes > 0)
      o.grid_byte_budget = size_t(grid_bytes);
    Context c;
    c.prepare(s, cutoff, o);
    int capacity = int(std::min<int64_t>(cap, 1 << 28));
    int *edges = c.array<int>("dump.edges", size_t(std::max(capacity, 1)) * 5);
    int *count = c.array<int>("dump.count", 1);
    execute(c, Dump{edges, count, capacity, c.internal_to_original});
    c.synchronize();
    int total = 0;
    check(cudaMemcpy(&total, count, 4, cudaMemcpyDeviceToHost));
    if (total > capacity)
      return total;
    std::vector<std::array<int, 5>> v(total);
    if (total)
      check(cudaMemcpy(v.data(), edges, size_t(total) * 20, cudaMemcpyDeviceToHost));
    std::sort(v.begin(), v.end());
    if (total)
      std::memcpy(out, v.data(), size_t(total) * 20);
    return total;
  } catch (const std::exception &e) {
    last_error = e.what();
    return -1;
  }
}
