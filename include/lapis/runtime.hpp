// Lapis L0 runtime: periodic geometry, device-built neighbour connectivity and reusable
// device workspaces.  Public API of the B200 build; the class and member names follow
// the reference interface (lapis/include/lapis/runtime.hpp:1-124) so callers and PairOps
// compile unchanged.  What differs is where the work runs: prepare() wraps, bins and
// enumerates neighbours on the device (no host pass over atoms) and leaves a
// receiver-major CSR edge list in HBM that every traversal of the call reuses.
#pragma once
#include <array>
#include <atomic>
#include <cstdint>
#include <cuda_runtime.h>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace lapis {
struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};
inline void check(cudaError_t e) {
  if (e != cudaSuccess)
    throw Error(cudaGetErrorString(e));
}
// Same enumerators and values as the reference (0 Auto, 1 BruteForce, 2 CellList).
enum class NeighborBackend { Auto, BruteForce, CellList };
struct Options {
  NeighborBackend backend = NeighborBackend::Auto;
  size_t grid_byte_budget = 64 * 1024 * 1024;
  int grid_to_atom_budget = 8;
};
struct Structure {
  int size = 0;
  const float *positions = nullptr; // Cartesian, N x 3, Angstrom
  const int *elements = nullptr;    // atomic numbers
  std::array<float, 9> cell{};      // lattice vectors are rows
  std::array<bool, 3> pbc{true, true, true};
};
struct Result {
  double energy = 0;
  std::vector<float> energies, forces;
  std::array<float, 9> virial{}; // -dE/d(strain), eV, row major
};
struct Diagnostics {
  NeighborBackend selected = NeighborBackend::BruteForce;
  std::array<int, 3> grid{1, 1, 1};
  int max_occupancy = 0, occupied_bins = 0;
  double mean_occupancy = 0, grid_candidates = 0, brute_candidates = 0;
  size_t allocated_bytes = 0, peak_bytes = 0;
  float device_ms = 0;
  std::string reason;
  long long edges = 0; // directed edges of the last call (B200 build addition)
  int launches = 0;     // kernels launched by the last call (B200 build addition)
  // How the last MH1 call ran its kernels (B200 build addition): "direct", "recorded" (captured
  // into a CUDA graph and launched) or "replayed" (the recorded graph launched again).
  std::string graph = "direct";
  std::vector<std::pair<std::string, float>> stages; // per-stage device ms when profiling
};
// Kernel launch counter of the calling thread (reset by Context::prepare).
int &launch_counter();
struct KernelResources {
  std::string name;
  int registers = 0, block_threads = 0, active_blocks_per_sm = 0;
  size_t static_shared = 0, dynamic_shared = 0;
};
struct Buffer {
  void *data = nullptr;
  size_t capacity = 0;
  Buffer() = default;
  Buffer(const Buffer &) = delete;
  Buffer &operator=(const Buffer &) = delete;
  ~Buffer() {
    if (data)
      cudaFree(data);
  }
  bool reserve(size_t bytes);
  template <class T> T *as() const { return static_cast<T *>(data); }
};
// Traversal parameters, passed by value to kernels.  Atom arrays are in the internal
// (bin-sorted) order.  The CSR lists, per internal receiver i, the directed edges
// [edge_offsets[i], edge_offsets[i+1]) with their sender, caller-frame image shift,
// float32 displacement x_j + shift.H - x_i and length.
struct DeviceGeometry {
  int n, grid[3], images[3];
  float h[9], cutoff2;
  const float *xyz;
  const int *elements, *bins, *offsets, *winding;
  int *status;
  NeighborBackend backend;
  const int *edge_offsets = nullptr;   // [n + 1]
  const int *edge_sender = nullptr;    // [E]
  const int *edge_shift = nullptr;     // [E][3]
  const float4 *edge_vector = nullptr; // [E] (dx, dy, dz, r)
  const float *edge_r2 = nullptr;      // [E] squared length compared against the cutoff
  const int *edge_reverse = nullptr;   // [E] index of the edge j <- i with the opposite shift
  long long edge_capacity = 0;
  // Rows of the CSR (B200 build addition): internal receivers [receiver_begin,
  // receiver_begin + receiver_count); all n atoms unless the context is partitioned.  In a
  // partitioned list an edge whose reverse lies outside these rows has edge_reverse -1.
  int receiver_begin = 0, receiver_count = 0;
};
struct WorkspaceSpec {
  size_t global_bytes = 0, scratch_bytes = 0, scratch_alignment = 16;
};
class Context {
  std::map<std::string, Buffer> buffers_;
  void *pinned_ = nullptr;
  size_t pinned_capacity_ = 0;
  const int *input_elements_ = nullptr; // device copy of the input-order atomic numbers

public:
  cudaStream_t stream{};
  cudaEvent_t start{}, stop{};
  DeviceGeometry geometry{};
  Diagnostics diagnostics;
  std::vector<KernelResources> resources;
  std::vector<int> original_elements;
  std::vector<int> batch_offsets; // prepared batch: first atom of each cell, plus the total
  int *internal_to_original = nullptr, *original_to_internal = nullptr;
  // Device-resident inputs: when set, prepare() reads positions/elements from these
  // device pointers instead of copying host arrays (the timed device-only path).
  const float *device_positions = nullptr;
  const int *device_elements = nullptr;
  // Receiver partition (B200 build addition, for domain decomposition): prepare() builds the
  // CSR rows of internal receivers [n part / parts, n (part + 1) / parts) only -- senders
  // still range over all atoms and images.  Default: all receivers.
  int part = 0, parts = 1;
  Context();
  ~Context();
  Context(const Context &) = delete;
  Context &operator=(const Context &) = delete;
  void *reserve(const std::string &name, size_t bytes);
  template <class T> T *array(const std::string &name, size_t count) {
    if (count > SIZE_MAX / sizeof(T))
      throw Error("Workspace byte count overflow");
    return static_cast<T *>(reserve(name, count * sizeof(T)));
  }
  void clear(void *p, size_t bytes) {
    if (bytes)
      check(cudaMemsetAsync(p, 0, bytes, stream));
  }
  void prepare(const Structure &, float, const Options &);
  // Reorders per-node energies/forces into input order and reduces energy and virial in
  // float64 on the device; node_virials is the per-node 3x3 virial [n][9].  When
  // e0_by_z (device, indexed by atomic number) is given, each atom's baseline energy is
  // added to its energy and to the total, in float64 for the total.
  Result finish(float *energies, float *forces, float *node_virials, const float *e0_by_z = nullptr);
  // Batch of independent periodic cells (B200 build addition, no reference counterpart):
  // one combined graph, atoms concatenated in input order (internal order = input order),
  // each cell wrapped with its own lattice and enumerated over its own atoms and images
  // (all-images enumeration; the edge set equals the single-cell one), one host sync.
  void prepare_batch(const std::vector<Structure> &cells, float cutoff, const Options &);
  // Per-cell results of a prepared batch: energies/virials reduced per cell in float64.
  std::vector<Result> finish_batch(float *energies, float *forces, float *node_virials,
                                   const float *e0_by_z = nullptr);
  void synchronize();
  int status_code(); // device status word (0 ok, 1 zero distance, 2 unknown element)
};
class Calculator {
  std::atomic_flag busy_ = ATOMIC_FLAG_INIT;

protected:
  // Batched evaluation hook: the default rejects batches (LJ and user calculators).
  virtual std::vector<Result> evaluate_batch();
  Context context_;
  Options options_;
  float cutoff_;
  virtual Result evaluate() = 0;

public:
  Calculator(float cutoff, Options options = {}) : options_(options), cutoff_(cutoff) {}
  virtual ~Calculator() = default;
  Result calculate(const Structure &);
  // Independent cells in one call (B200 build addition): same results as calculate() per
  // cell up to float32 summation order; evaluated in sub-batches of at most
  // kBatchAtoms atoms so the workspace stays bounded.  Single-flight like calculate().
  static constexpr int kBatchAtoms = 65536;
  std::vector<Result> calculate_batch(const std::vector<Structure> &cells);
  const Diagnostics &diagnostics() const { return context_.diagnostics; }
  const std::vector<KernelResources> &resources() const { return context_.resources; }
  Context &context() { return context_; }
};
} // namespace lapis
