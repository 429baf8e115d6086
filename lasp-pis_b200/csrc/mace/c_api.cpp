// C ABI of the B200 build (mace/include/mace/c_api.h).  Same contract as the reference's
// mace/src/c_api.cpp:18-98: exceptions become -1 / NULL plus a thread-local message, null
// result pointers are accepted only for n == 0, outputs are caller-owned in input order.
// Handles remember the CUDA device they were created on and make it current per call.
#include "mace/c_api.h"
#include "mace/mh1.hpp"
#include "model.hpp"
#include <algorithm>
#include <array>
#include <cstring>
#include <climits>
#include <sstream>
#include <vector>

using namespace lapis;
using mace::MH1;
namespace {
thread_local std::string error;
} // namespace
namespace lapis {
void set_c_api_error(const std::string &message) { error = message; }
} // namespace lapis
namespace {

struct Handle {
  int device = 0;
  std::unique_ptr<MH1> model;
};

Options options(int b) {
  if (b < 0 || b > 2)
    throw Error("Invalid backend");
  Options o;
  o.backend = NeighborBackend(b);
  return o;
}

struct DeviceScope {
  int previous = -1;
  explicit DeviceScope(int device) {
    check(cudaGetDevice(&previous));
    if (previous != device)
      check(cudaSetDevice(device));
  }
  ~DeviceScope() {
    int now = -1;
    if (previous >= 0 && cudaGetDevice(&now) == cudaSuccess && now != previous)
      cudaSetDevice(previous);
  }
};

Handle *create(const char *path, int b, const char *head, int device) {
  if (!path)
    throw Error("Null archive path");
  auto h = std::make_unique<Handle>();
  if (device < 0)
    check(cudaGetDevice(&h->device));
  else
    h->device = device;
  DeviceScope scope(h->device);
  h->model = std::make_unique<MH1>(path, options(b), head ? head : "");
  return h.release();
}

long long dump_edges(Context &ctx, int *out, long long capacity) {
  // The prepared CSR rows: receivers [receiver_begin, receiver_begin + receiver_count) of the
  // internal order (all atoms, or this rank's atoms in a domain-decomposed handle).
  const auto &g = ctx.geometry;
  long long E = g.edge_capacity;
  int n = g.n, rows = g.receiver_count, r0 = g.receiver_begin;
  std::vector<int> row(static_cast<size_t>(rows) + 1), sender(static_cast<size_t>(E)),
      shift(static_cast<size_t>(E) * 3), i2o(static_cast<size_t>(n));
  if (n) {
    check(cudaMemcpy(row.data(), g.edge_offsets, (size_t(rows) + 1) * 4, cudaMemcpyDeviceToHost));
    check(cudaMemcpy(i2o.data(), ctx.internal_to_original, size_t(n) * 4, cudaMemcpyDeviceToHost));
  }
  if (E) {
    check(cudaMemcpy(sender.data(), g.edge_sender, size_t(E) * 4, cudaMemcpyDeviceToHost));
    check(cudaMemcpy(shift.data(), g.edge_shift, size_t(E) * 12, cudaMemcpyDeviceToHost));
  }
  std::vector<std::array<int, 5>> edges(static_cast<size_t>(E));
  for (int w = 0; w < rows; ++w)
    for (int e = row[w]; e < row[w + 1]; ++e)
      edges[e] = {i2o[r0 + w], i2o[sender[e]], shift[3 * e], shift[3 * e + 1], shift[3 * e + 2]};
  std::sort(edges.begin(), edges.end());
  long long copy = std::min(E, std::max(capacity, 0ll));
  if (copy)
    std::memcpy(out, edges.data(), size_t(copy) * 20);
  return E;
}

int calculate(void *handle, int n, const float *xyz, const int *z, const float *cell, double *energy,
              float *per_atom, float *force, float *virial, bool on_device) {
  try {
    error.clear();
    if (!handle || !cell || !energy || !virial || (n && (!per_atom || !force)))
      throw Error("Null calculator or result pointer");
    if (n < 0)
      throw Error("Invalid atom count or cutoff");
    auto *h = static_cast<Handle *>(handle);
    DeviceScope scope(h->device);
    Structure s;
    s.size = n;
    s.positions = on_device ? nullptr : xyz;
    s.elements = on_device ? nullptr : z;
    std::copy(cell, cell + 9, s.cell.begin());
    auto &ctx = h->model->context();
    if (on_device && n && (!xyz || !z))
      throw Error("Null structure data");
    ctx.device_positions = on_device ? xyz : nullptr;
    ctx.device_elements = on_device ? z : nullptr;
    struct Reset {
      Context &c;
      ~Reset() {
        c.device_positions = nullptr;
        c.device_elements = nullptr;
      }
    } reset{ctx};
    auto r = h->model->calculate(s);
    *energy = r.energy;
    std::copy(r.energies.begin(), r.energies.end(), per_atom);
    std::copy(r.forces.begin(), r.forces.end(), force);
    std::copy(r.virial.begin(), r.virial.end(), virial);
    return 0;
  } catch (const std::exception &e) {
    error = e.what();
    return -1;
  }
}
} // namespace

extern "C" {
void *mace_create_mh1(const char *path, int b) { return mace_create_mh1_head(path, b, nullptr); }

int mace_check_model(const char *path, const char *head) {
  try {
    error.clear();
    if (!path)
      throw Error("Null archive path");
    mace::ModelData data;
    data.validate(path, head ? head : "");
    return 0;
  } catch (const std::exception &e) {
    error = e.what();
    return -1;
  }
}

void *mace_create_mh1_head(const char *path, int b, const char *head) {
  try {
    error.clear();
    return create(path, b, head, -1);
  } catch (const std::exception &e) {
    error = e.what();
    return nullptr;
  }
}

void *mace_create_mh1_device(const char *path, int b, int device) {
  return mace_create_mh1_device_head(path, b, nullptr, device);
}

void *mace_create_mh1_device_head(const char *path, int b, const char *head, int device) {
  try {
    error.clear();
    if (device < 0)
      throw Error("Invalid device");
    return create(path, b, head, device);
  } catch (const std::exception &e) {
    error = e.what();
    return nullptr;
  }
}

void *mace_create_mh1_domain(const char *path, int b, int device, int rank, int world, const void *nccl_id) {
  try {
    error.clear();
    if (device < 0)
      throw Error("Invalid device");
    if (!nccl_id)
      throw Error("Null NCCL id");
    auto *h = static_cast<Handle *>(create(path, b, nullptr, device));
    try {
      DeviceScope scope(h->device);
      h->model->set_domain(std::make_shared<lapis::Domain>(rank, world, nccl_id));
    } catch (...) {
      mace_destroy(h);
      throw;
    }
    return h;
  } catch (const std::exception &e) {
    error = e.what();
    return nullptr;
  }
}

int mace_nccl_unique_id(void *out) {
  try {
    error.clear();
    if (!out)
      throw Error("Null output");
    auto id = lapis::nccl_unique_id();
    std::copy(id.begin(), id.end(), static_cast<char *>(out));
    return 0;
  } catch (const std::exception &e) {
    error = e.what();
    return -1;
  }
}

void mace_destroy(void *handle) {
  auto *h = static_cast<Handle *>(handle);
  if (!h)
    return;
  int previous = -1;
  cudaGetDevice(&previous);
  cudaSetDevice(h->device);
  delete h;
  if (previous >= 0)
    cudaSetDevice(previous);
}

const char *mace_last_error() { return error.c_str(); }

int mace_calculate(void *h, int n, const float *xyz, const int *z, const float *cell, double *energy,
                   float *per_atom, float *force, float *virial) {
  return calculate(h, n, xyz, z, cell, energy, per_atom, force, virial, false);
}

int mace_calculate_device(void *h, int n, const float *xyz, const int *z, const float *cell, double *energy,
                          float *per_atom, float *force, float *virial) {
  return calculate(h, n, xyz, z, cell, energy, per_atom, force, virial, true);
}

int mace_calculate_batch(void *handle, int count, const int *sizes, const float *xyz, const int *z,
                         const float *cells, double *energies, float *per_atom, float *force, float *virial) {
  try {
    error.clear();
    if (!handle || count < 0 || (count && (!sizes || !cells || !energies || !virial)))
      throw Error("Null calculator or result pointer");
    long long total = 0;
    for (int c = 0; c < count; ++c) {
      if (sizes[c] < 0)
        throw Error("Invalid atom count or cutoff");
      total += sizes[c];
    }
    if (total > INT_MAX / 16)
      throw Error("Invalid atom count or cutoff");
    if (total && (!xyz || !z || !per_atom || !force))
      throw Error("Null structure data");
    auto *h = static_cast<Handle *>(handle);
    DeviceScope scope(h->device);
    std::vector<Structure> part(static_cast<size_t>(count));
    long long first = 0;
    for (int c = 0; c < count; ++c) {
      Structure &s = part[c];
      s.size = sizes[c];
      s.positions = sizes[c] ? xyz + 3 * first : nullptr;
      s.elements = sizes[c] ? z + first : nullptr;
      std::copy(cells + 9 * size_t(c), cells + 9 * size_t(c) + 9, s.cell.begin());
      first += sizes[c];
    }
    auto results = h->model->calculate_batch(part);
    first = 0;
    for (int c = 0; c < count; ++c) {
      const auto &r = results[c];
      energies[c] = r.energy;
      std::copy(r.energies.begin(), r.energies.end(), per_atom + first);
      std::copy(r.forces.begin(), r.forces.end(), force + 3 * first);
      std::copy(r.virial.begin(), r.virial.end(), virial + 9 * size_t(c));
      first += sizes[c];
    }
    return 0;
  } catch (const std::exception &e) {
    error = e.what();
    return -1;
  }
}

long long mace_last_edges(void *handle, int *out, long long capacity) {
  try {
    error.clear();
    if (!handle || (capacity > 0 && !out))
      throw Error("Null calculator or result pointer");
    auto *h = static_cast<Handle *>(handle);
    DeviceScope scope(h->device);
    return dump_edges(h->model->context(), out, capacity);
  } catch (const std::exception &e) {
    error = e.what();
    return -1;
  }
}

long long lapis_neighbor_edges(int n, const float *xyz, const float *cell, float cutoff, int backend,
                               long long grid_bytes, int *out, long long capacity) {
  try {
    error.clear();
    if (!cell || (capacity > 0 && !out))
      throw Error("Null structure data");
    Options o = options(backend);
    if (grid_bytes > 0)
      o.grid_byte_budget = size_t(grid_bytes);
    std::vector<int> z(static_cast<size_t>(std::max(n, 0)), 1);
    Structure s;
    s.size = n;
    s.positions = xyz;
    s.elements = z.data();
    std::copy(cell, cell + 9, s.cell.begin());
    Context ctx;
    ctx.prepare(s, cutoff, o);
    ctx.synchronize();
    return dump_edges(ctx, out, capacity);
  } catch (const std::exception &e) {
    error = e.what();
    return -1;
  }
}

int mace_profile(void *handle, int enable) {
  try {
    error.clear();
    if (!handle)
      throw Error("Null calculator or result pointer");
    static_cast<Handle *>(handle)->model->set_profiling(enable != 0);
    return 0;
  } catch (const std::exception &e) {
    error = e.what();
    return -1;
  }
}

int mace_diagnostics(void *handle, char *buffer, size_t capacity) {
  try {
    if (!handle || !buffer)
      throw Error("Null diagnostics pointer");
    auto *h = static_cast<Handle *>(handle);
    auto &d = h->model->diagnostics();
    std::ostringstream s;
    s << "{\"backend\":\"" << (d.selected == NeighborBackend::CellList ? "CellList" : "BruteForce")
      << "\",\"grid\":[" << d.grid[0] << "," << d.grid[1] << "," << d.grid[2] << "],\"reason\":\"" << d.reason
      << "\",\"max_occupancy\":" << d.max_occupancy << ",\"occupied_bins\":" << d.occupied_bins
      << ",\"mean_occupancy\":" << d.mean_occupancy << ",\"grid_candidates\":" << d.grid_candidates
      << ",\"brute_candidates\":" << d.brute_candidates << ",\"context_bytes\":" << d.allocated_bytes
      << ",\"context_peak_bytes\":" << d.peak_bytes << ",\"parameter_bytes\":" << h->model->parameter_bytes()
      << ",\"device_ms\":" << d.device_ms << ",\"edges\":" << d.edges << ",\"device\":" << h->device
      << ",\"launches\":" << d.launches << ",\"graph\":\"" << d.graph << "\",\"stages\":[";
    for (size_t k = 0; k < d.stages.size(); ++k)
      s << (k ? "," : "") << "[\"" << d.stages[k].first << "\"," << d.stages[k].second << "]";
    s << "],\"kernels\":[";
    bool first = true;
    for (auto &r : h->model->resources()) {
      if (!first)
        s << ",";
      first = false;
      s << "{\"name\":\"" << r.name << "\",\"registers\":" << r.registers << ",\"threads\":" << r.block_threads
        << ",\"static_shared\":" << r.static_shared << ",\"dynamic_shared\":" << r.dynamic_shared
        << ",\"blocks_per_sm\":" << r.active_blocks_per_sm << "}";
    }
    s << "]}";
    auto str = s.str();
    if (str.size() + 1 > capacity)
      throw Error("Diagnostics buffer too small");
    std::memcpy(buffer, str.c_str(), str.size() + 1);
    return 0;
  } catch (const std::exception &e) {
    error = e.what();
    return -1;
  }
}
}
