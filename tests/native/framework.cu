// Native test of the Lapis PairOp extension API and its Lennard-Jones example on the GPU.
// Checks the semantics the reference's lapis/tests/framework.cu pins (lines 158-258):
// edge-set semantics through an edge-collecting operation (tile boundaries and partial
// tiles, inclusive cutoff, self-images, multidimensional blocks), LJ finite differences and
// momentum, workspace reuse and repeatability, the single-flight rule, resource rejection
// and geometry errors.  Prints one line per group; exits 1 on the first failure.
#include <lapis/lj.hpp>
#include <lapis/pair.cuh>

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdio>
#include <future>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

using namespace lapis;

static void require(bool ok, const char *what) {
  if (!ok)
    throw std::runtime_error(what);
}

// Appends (receiver, sender, sx, sy, sz) of every edge it sees, in original atom ids.
template <int Threads, int Tile, bool Shaped> struct CollectOp {
  static constexpr int threads = Threads, tile_edges = Tile, scratch_alignment = 32;
  static const char *name() { return Shaped ? "collect_shaped" : "collect"; }
  struct State {
    int seen;
  };
  int *out, *count, *to_original;
  int capacity;
  WorkspaceSpec plan(int) const { return {0, 64, 32}; }
  void setup(Context &, void *) {}
  void postprocess(Context &, void *) {}
  __device__ void prepare(int, State &s, void *) { s.seen = 0; }
  template <class TileT> __device__ void consume(int i, const TileT &tile, State &s, void *) {
    int t = thread_rank();
    for (int e = t; e < tile.size(); e += threads) {
      int slot = atomicAdd(count, 1);
      if (slot < capacity) {
        int3 sh = tile.shift(e);
        int *o = out + 5 * slot;
        o[0] = to_original[i];
        o[1] = to_original[tile.sender(e)];
        o[2] = sh.x, o[3] = sh.y, o[4] = sh.z;
      }
    }
    s.seen += tile.size();
  }
  __device__ void finalize(int, State &, void *) {}
};
// Shaped variant: declares a two-row block; everything else equal.
template <int Threads, int Tile> struct ShapedCollect : CollectOp<Threads, Tile, true> {
  static dim3 block_shape() { return dim3(Threads / 2, 2, 1); }
};

struct ExcessiveOp {
  static constexpr int threads = 32, tile_edges = 4, scratch_alignment = 16;
  static const char *name() { return "excessive"; }
  struct State {};
  WorkspaceSpec plan(int) const { return {0, size_t(4) << 20, 16}; }
  void setup(Context &, void *) {}
  void postprocess(Context &, void *) {}
  __device__ void prepare(int, State &, void *) {}
  template <class T> __device__ void consume(int, const T &, State &, void *) {}
  __device__ void finalize(int, State &, void *) {}
};

using Edge = std::array<int, 5>;

template <class Op> static std::vector<Edge> collect_with(const Structure &s, float cutoff, Options o) {
  Context c;
  c.prepare(s, cutoff, o);
  long long E = c.geometry.edge_capacity;
  int *buf = c.array<int>("collect.out", size_t(std::max<long long>(E, 1)) * 5);
  int *count = c.array<int>("collect.count", 1);
  c.clear(count, sizeof(int));
  Op op{};
  op.out = buf, op.count = count, op.to_original = c.internal_to_original, op.capacity = int(E);
  execute(c, op);
  c.synchronize();
  int n = 0;
  check(cudaMemcpy(&n, count, sizeof(int), cudaMemcpyDeviceToHost));
  require(n == E, "operation saw a different edge count than the traversal");
  std::vector<Edge> edges(n);
  if (n)
    check(cudaMemcpy(edges.data(), buf, size_t(n) * 5 * sizeof(int), cudaMemcpyDeviceToHost));
  std::sort(edges.begin(), edges.end());
  return edges;
}
static std::vector<Edge> collect(const Structure &s, float cutoff, Options o = {}) {
  return collect_with<CollectOp<32, 7, false>>(s, cutoff, o);
}

// Double-precision periodic reference: every image within the cutoff, inclusive, (i, i, 0)
// excluded, shift = image of the sender.
static std::vector<Edge> brute(const Structure &s, float cutoff, int images) {
  std::vector<Edge> out;
  for (int i = 0; i < s.size; ++i)
    for (int j = 0; j < s.size; ++j)
      for (int x = -images; x <= images; ++x)
        for (int y = -images; y <= images; ++y)
          for (int z = -images; z <= images; ++z) {
            if (i == j && !x && !y && !z)
              continue;
            double r2 = 0;
            for (int k = 0; k < 3; ++k) {
              double d = s.positions[3 * j + k] + x * s.cell[k] + y * s.cell[3 + k] + z * s.cell[6 + k] -
                         s.positions[3 * i + k];
              r2 += d * d;
            }
            if (r2 <= double(cutoff) * cutoff)
              out.push_back({i, j, x, y, z});
          }
  std::sort(out.begin(), out.end());
  return out;
}

// Blocks inside evaluate() until released, to test the single-flight rule.
class HeldCalculator final : public Calculator {
  std::promise<void> &entered_;
  std::shared_future<void> release_;
  Result evaluate() override {
    entered_.set_value();
    release_.wait();
    size_t n = size_t(context_.geometry.n);
    float *e = context_.array<float>("h.e", n), *f = context_.array<float>("h.f", 3 * n),
          *v = context_.array<float>("h.v", 9 * n);
    context_.clear(e, n * sizeof(float));
    context_.clear(f, 3 * n * sizeof(float));
    context_.clear(v, 9 * n * sizeof(float));
    return context_.finish(e, f, v);
  }

public:
  HeldCalculator(std::promise<void> &entered, std::shared_future<void> release)
      : Calculator(2.5f), entered_(entered), release_(std::move(release)) {}
};

int main() {
  try {
    // ---- edge semantics against a float64 brute-force enumeration ----
    {
      std::vector<float> x = {0.1f, 0.2f, 0.3f, 1.9f, 0.4f, 0.1f, 0.7f, 2.6f, 1.2f, 2.2f, 2.1f, 2.8f, 1.1f, 1.3f, 0.9f};
      std::vector<int> z(5, 6);
      Structure s;
      s.size = 5;
      s.positions = x.data();
      s.elements = z.data();
      s.cell = {3.1f, 0, 0, 0.4f, 3.3f, 0, -0.2f, 0.3f, 3.0f};
      auto ref = brute(s, 2.5f, 2);
      for (int backend = 0; backend < 3; ++backend) {
        Options o;
        o.backend = NeighborBackend(backend);
        if (backend == 2)
          continue; // plane heights below the cutoff: the explicit cell list is rejected below
        require(collect(s, 2.5f, o) == ref, "edge multiset differs from the float64 enumeration");
      }
      require(collect_with<ShapedCollect<64, 5>>(s, 2.5f, {}) == ref, "shaped block edge multiset mismatch");
      require(collect_with<CollectOp<128, 128, false>>(s, 2.5f, {}) == ref, "wide tile edge multiset mismatch");
      std::printf("edge semantics (self-images, shapes, tiles) passed (%zu edges)\n", ref.size());
    }
    // ---- tile boundaries: every pair within the cutoff ----
    for (int count : {1, 2, 7, 8, 15, 16, 17, 33, 128, 129, 145}) {
      std::vector<float> x(size_t(count) * 3, 1.f);
      std::vector<int> z(count, 1);
      for (int i = 0; i < count; ++i)
        x[3 * i] += i * 1e-4f;
      Structure q;
      q.size = count;
      q.positions = x.data();
      q.elements = z.data();
      q.cell = {8, 0, 0, 0, 8, 0, 0, 0, 8};
      auto edges = collect(q, .5f);
      require(edges.size() == size_t(count) * (count - 1), "tile boundary edge count mismatch");
      require(std::adjacent_find(edges.begin(), edges.end()) == edges.end(), "duplicate edge");
    }
    std::printf("tile boundaries passed\n");
    // ---- inclusive cutoff ----
    {
      float x[6] = {0, 0, 0, 2.5f, 0, 0};
      int z[2] = {1, 1};
      Structure q;
      q.size = 2;
      q.positions = x;
      q.elements = z;
      q.cell = {8, 0, 0, 0, 8, 0, 0, 0, 8};
      require(collect(q, 2.5f).size() == 2, "inclusive cutoff rejected");
      x[3] = std::nextafter(2.5f, 3.f);
      require(collect(q, 2.5f).empty(), "above cutoff accepted");
      x[3] = std::nextafter(2.5f, 2.f);
      require(collect(q, 2.5f).size() == 2, "below cutoff rejected");
      Options grid;
      grid.backend = NeighborBackend::CellList;
      q.cell = {1, 0, 0, 0, 1, 0, 0, 0, 1};
      bool rejected = false;
      try {
        collect(q, 2.5f, grid);
      } catch (const Error &) {
        rejected = true;
      }
      require(rejected, "invalid explicit grid accepted");
      std::printf("inclusive cutoff passed\n");
    }
    // ---- Lennard-Jones: finite differences, momentum, reuse, repeat ----
    float xyz[6] = {.2f, .3f, .4f, 1.4f, .3f, .4f};
    int zs[2] = {18, 18};
    Structure s;
    s.size = 2;
    s.positions = xyz;
    s.elements = zs;
    s.cell = {8, 0, 0, 0, 8, 0, 0, 0, 8};
    LennardJones lj;
    auto a = lj.calculate(s);
    float step = .001f;
    xyz[3] = 1.4f + step;
    double ep = lj.calculate(s).energy;
    xyz[3] = 1.4f - step;
    double em = lj.calculate(s).energy;
    xyz[3] = 1.4f;
    require(std::abs(a.forces[3] + (ep - em) / (2 * step)) < .001, "LJ finite difference mismatch");
    require(std::abs(a.forces[0] + a.forces[3]) < 1e-6, "LJ momentum mismatch");
    auto capacity = lj.diagnostics().allocated_bytes;
    auto b = lj.calculate(s);
    require(capacity == lj.diagnostics().allocated_bytes, "workspace not reused");
    require(a.energy == b.energy, "repeat mismatch");
    std::printf("LJ derivatives, momentum, reuse and repeat passed (E = %.6f)\n", a.energy);
    // ---- single flight ----
    {
      std::promise<void> entered, release;
      auto ready = entered.get_future();
      HeldCalculator held(entered, release.get_future().share());
      std::exception_ptr worker_error;
      std::thread worker([&]() {
        try {
          held.calculate(s);
        } catch (...) {
          worker_error = std::current_exception();
        }
      });
      ready.wait();
      bool rejected = false;
      try {
        held.calculate(s);
      } catch (const Error &e) {
        rejected = std::string(e.what()).find("single-flight") != std::string::npos;
      }
      release.set_value();
      worker.join();
      if (worker_error)
        std::rethrow_exception(worker_error);
      require(rejected, "concurrent call not rejected");
      std::printf("single-flight passed\n");
    }
    // ---- resource limits and geometry errors ----
    {
      Context c;
      c.prepare(s, 2.5f, {});
      bool rejected = false;
      try {
        execute(c, ExcessiveOp{});
      } catch (const Error &) {
        rejected = true;
      }
      require(rejected, "excessive scratch accepted");
    }
    s.cell[8] = 0;
    bool threw = false;
    try {
      lj.calculate(s);
    } catch (const Error &) {
      threw = true;
    }
    require(threw, "singular cell accepted");
    std::printf("resource limits and geometry errors passed\n");
    return 0;
  } catch (const std::exception &e) {
    std::fprintf(stderr, "FAILED: %s\n", e.what());
    return 1;
  }
}
