// Model loading for the B200 build: a PWMH1001 archive, or an MH1 PyTorch ZIP checkpoint
// converted to one on the host first (checkpoint.hpp; mace/src/mh1.cu:626-627).
//
// Record format and validation rules follow the reference loader (mace/src/mh1.cu:626-734,
// mace/src/weights.cpp:305-317): magic, record count <= 10000, name length <= 1024, record
// size <= 512 MiB and a multiple of 4, unique names, finite float records, shape checks
// per tensor, linear path bounds, tensor-product and polynomial index bounds.  Error
// messages are the reference's so callers see the same failures.  Radial matrices are
// transposed at load (as the reference does) for coalesced per-unit reads, and the
// tensor-product terms are mapped onto the term table compiled into the edge kernels.
#include "model.hpp"
#include "checkpoint.hpp"
#include "product_table.h"
#include <cuda_fp16.h>
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>

namespace mace {
using lapis::Error;
using lapis::check;

Device::~Device() {
  for (void *p : allocations)
    if (host_only)
      std::free(p);
    else
      cudaFree(p);
}

float *Device::upload(const void *data, size_t bytes) {
  void *p = nullptr;
  if (host_only) {
    p = std::malloc(bytes ? bytes : 4);
    if (!p)
      throw Error("out of host memory");
    allocations.push_back(p);
    if (bytes)
      std::memcpy(p, data, bytes);
    return static_cast<float *>(p);
  }
  check(cudaMalloc(&p, bytes ? bytes : 4));
  allocations.push_back(p);
  if (bytes)
    check(cudaMemcpy(p, data, bytes, cudaMemcpyHostToDevice));
  return static_cast<float *>(p);
}

void ModelData::validate(const std::string &path, const std::string &head) {
  if (!device.allocations.empty())
    throw Error("validate() needs a fresh model");
  device.host_only = true;
  load(path, head);
}

// w 2^exp = hi + lo: hi = round_fp16(w 2^exp), lo = round_fp16(w 2^exp - hi) (the remainder
// is exact in fp32); exp brings the largest |w| into [2^14, 2^15), so every weight down to
// 2^-17 of the largest keeps 22 significant bits in normal fp16 numbers.
int split_f16(const float *w, size_t count, uint16_t *hi, uint16_t *lo) {
  float m = 0.f;
  for (size_t k = 0; k < count; ++k)
    m = std::max(m, std::fabs(w[k]));
  int exp = 0;
  if (m > 0.f) {
    int ex = 0;
    std::frexp(m, &ex); // m = f 2^ex, f in [0.5, 1)
    exp = std::min(126, std::max(-126, 15 - ex));
  }
  float scale = std::ldexp(1.f, exp);
  for (size_t k = 0; k < count; ++k) {
    float x = w[k] * scale;
    __half h = __float2half_rn(x);
    __half l = __float2half_rn(x - __half2float(h));
    std::memcpy(hi + k, &h, 2);
    std::memcpy(lo + k, &l, 2);
  }
  return exp;
}

namespace {
struct Archive {
  std::map<std::string, std::vector<char>> records;
  template <class T> std::vector<T> get(const std::string &key) const {
    auto it = records.find(key);
    if (it == records.end() || it->second.size() % sizeof(T))
      throw Error("Invalid MH1 tensor " + key);
    std::vector<T> out(it->second.size() / sizeof(T));
    std::memcpy(out.data(), it->second.data(), it->second.size());
    return out;
  }
  void require_size(const std::string &key, size_t count, size_t item = 4) const {
    auto it = records.find(key);
    if (it == records.end() || it->second.size() != count * item)
      throw Error("Invalid MH1 tensor size: " + key);
  }
  bool has(const std::string &key) const { return records.count(key) != 0; }
};

bool ends_with(const std::string &s, const char *t) {
  size_t n = std::strlen(t);
  return s.size() >= n && s.compare(s.size() - n, n, t) == 0;
}

Archive read_archive(const std::string &path, const std::string &head) {
  std::ifstream in(path, std::ios::binary | std::ios::ate);
  if (!in)
    throw Error("Cannot open MH1 archive: " + path);
  auto size = in.tellg();
  const bool zip = size >= 4 && [&] {
    char magic[4];
    in.seekg(0);
    return in.read(magic, 4) && std::memcmp(magic, "PK\x03\x04", 4) == 0;
  }();
  std::string bytes;
  if (zip) {
    // An original checkpoint: convert it for the requested head (the ZIP layer enforces
    // its own 2 GiB bound).
    if (uint64_t(size) > (uint64_t(1) << 31))
      throw Error("checkpoint: archive exceeds 2 GiB limit");
    std::vector<char> file(static_cast<size_t>(size));
    in.seekg(0);
    if (!in.read(file.data(), std::streamsize(file.size())))
      throw Error("cannot read MH1 archive: " + path);
    try {
      bytes = convert_checkpoint(std::move(file), head);
    } catch (const Error &) {
      throw;
    } catch (const std::exception &e) {
      throw Error(e.what());
    }
  } else {
    if (!head.empty())
      throw Error("unsupported MH1 checkpoint: head selection requires an original checkpoint; an archive "
                  "already contains one head");
    if (size < 0 || uint64_t(size) >= (uint64_t(1) << 31))
      throw Error("unsupported MH1 checkpoint: archive size");
    bytes.assign(size_t(size), '\0');
    in.clear();
    in.seekg(0);
    if (!in.read(bytes.data(), std::streamsize(bytes.size())))
      throw Error("cannot read MH1 archive: " + path);
  }
  std::istringstream s(bytes, std::ios::binary);
  char magic[8]{};
  s.read(magic, 8);
  if (!s || std::memcmp(magic, "PWMH1001", 8))
    throw Error("Invalid MH1 archive magic");
  uint32_t count = 0;
  s.read(reinterpret_cast<char *>(&count), 4);
  if (!s || count == 0 || count > 10000)
    throw Error("Invalid MH1 tensor count");
  Archive a;
  for (uint32_t k = 0; k < count; ++k) {
    uint32_t len = 0;
    uint64_t bytes_n = 0;
    s.read(reinterpret_cast<char *>(&len), 4);
    s.read(reinterpret_cast<char *>(&bytes_n), 8);
    if (!s || len > 1024 || !len || bytes_n > 512ull * 1024 * 1024)
      throw Error("Invalid MH1 archive record");
    std::string name(len, '\0');
    s.read(name.data(), len);
    if (a.records.count(name))
      throw Error("Duplicate MH1 tensor");
    auto &t = a.records[name];
    t.resize(bytes_n);
    s.read(t.data(), std::streamsize(bytes_n));
    if (!s)
      throw Error("Truncated MH1 archive");
    bool indices = name == "atomic_numbers" || ends_with(name, ".dims") || ends_with(name, ".paths") ||
                   ends_with(name, ".terms");
    if (bytes_n % 4)
      throw Error("Invalid MH1 tensor byte alignment: " + name);
    if (!indices)
      for (size_t i = 0; i < bytes_n; i += 4) {
        float v;
        std::memcpy(&v, t.data() + i, 4);
        if (!std::isfinite(v))
          throw Error("Nonfinite MH1 tensor: " + name);
      }
  }
  return a;
}

std::vector<float> transposed(const std::vector<float> &a, int rows, int cols, const std::string &key) {
  if (a.size() != size_t(rows) * cols)
    throw Error("Invalid radial matrix dimensions: " + key);
  std::vector<float> b(a.size());
  for (int i = 0; i < rows; ++i)
    for (int j = 0; j < cols; ++j)
      b[size_t(j) * rows + i] = a[size_t(i) * cols + j];
  return b;
}
} // namespace

void ModelData::load(const std::string &path, const std::string &head) {
  Archive a = read_archive(path, head);
  auto up = [&](const std::vector<float> &v) {
    bytes += v.size() * 4;
    return device.upload(v.data(), v.size() * 4);
  };
  // fp16 split planes of a K-major matrix for the tensor-core GEMM.
  auto up_split = [&](const float *w, size_t count) {
    std::vector<uint16_t> hi(count), lo(count);
    TCMatrix m;
    m.exp = split_f16(w, count, hi.data(), lo.data());
    bytes += count * 4;
    m.hi = reinterpret_cast<const uint16_t *>(device.upload(hi.data(), count * 2));
    m.lo = reinterpret_cast<const uint16_t *>(device.upload(lo.data(), count * 2));
    return m;
  };
  auto c = a.get<float>("constants");
  if (c.size() != 14 || c[0] != 6)
    throw Error("Unsupported MH1 constants");
  std::copy(c.begin(), c.end(), constants);
  constants_dev = up(c);
  auto zs = a.get<int>("atomic_numbers");
  species = int(zs.size());
  if (species < 1 || species > 118)
    throw Error("Invalid MH1 element count");
  a.require_size("embedding", size_t(species) * 512);
  a.require_size("bessel", 10);
  a.require_size("radii", 119);
  a.require_size("zbl.radii", 119);
  a.require_size("zbl.c", 4);
  auto e0 = a.get<float>("e0");
  if (e0.size() != zs.size())
    throw Error("Invalid atomic energy table");
  std::vector<int> lk(119, -1);
  std::vector<float> e0z(119, 0.f);
  for (size_t k = 0; k < zs.size(); ++k) {
    if (zs[k] < 1 || zs[k] > 118 || lk[zs[k]] >= 0)
      throw Error("Invalid MH1 element map");
    lk[zs[k]] = int(k);
    e0z[zs[k]] = e0[k];
  }
  lookup = reinterpret_cast<const int *>(device.upload(lk.data(), 119 * 4));
  e0_z = up(e0z);
  embedding = up(a.get<float>("embedding"));
  bessel = up(a.get<float>("bessel"));
  radii = up(a.get<float>("radii"));
  zbl_radii = up(a.get<float>("zbl.radii"));
  zbl_c = up(a.get<float>("zbl.c"));
  auto get_linear = [&](const std::string &key, int input, int output) {
    auto dims = a.get<int>(key + ".dims");
    if (dims.size() != 2 || dims[0] != input || dims[1] != output)
      throw Error("Unsupported MH1 linear dimensions: " + key);
    auto raw = a.get<int>(key + ".paths");
    if (raw.size() % 6)
      throw Error("Invalid MH1 tensor " + key + ".paths");
    auto w = a.get<float>(key + ".weight");
    Linear l;
    l.input = input;
    l.output = output;
    for (size_t k = 0; k < raw.size(); k += 6) {
      LinearPath p{raw[k], raw[k + 1], raw[k + 2], raw[k + 3], raw[k + 4], raw[k + 5]};
      if (p.in_offset < 0 || p.out_offset < 0 || p.in_mul <= 0 || p.out_mul <= 0 || p.in_mul > 2048 ||
          p.out_mul > 2048 || p.dim < 1 || p.dim > 7 || p.weight_offset < 0 ||
          int64_t(p.in_offset) + int64_t(p.in_mul) * p.dim > input ||
          int64_t(p.out_offset) + int64_t(p.out_mul) * p.dim > output ||
          size_t(p.weight_offset) + size_t(p.in_mul) * p.out_mul > w.size())
        throw Error("Invalid linear path: " + key);
      l.paths.push_back(p);
    }
    l.weight = up(w);
    for (const auto &p : l.paths) {
      TCWeights t;
      if (tc_gemm_supported(p.out_mul, p.in_mul) && tc_gemm_supported(p.in_mul, p.out_mul)) {
        size_t cnt = size_t(p.in_mul) * p.out_mul;
        const float *src = w.data() + p.weight_offset;
        std::vector<float> wt(cnt);
        for (int i = 0; i < p.in_mul; ++i)
          for (int o = 0; o < p.out_mul; ++o)
            wt[size_t(o) * p.in_mul + i] = src[size_t(i) * p.out_mul + o];
        t.fwd = up_split(wt.data(), cnt);
        t.bwd = up_split(src, cnt);
      }
      l.tc.push_back(t);
    }
    return l;
  };
  auto get_radial = [&](const std::string &key, int depth, int outputs) {
    a.require_size(key + ".source", size_t(species) * 64);
    a.require_size(key + ".target", size_t(species) * 64);
    for (int k = 0; k < depth; ++k) {
      a.require_size(key + "." + std::to_string(k * 3) + ".weight", k ? 64 * 64 : 64 * 1034);
      a.require_size(key + "." + std::to_string(k * 3) + ".bias", 64);
      a.require_size(key + "." + std::to_string(k * 3 + 1) + ".weight", 64);
      a.require_size(key + "." + std::to_string(k * 3 + 1) + ".bias", 64);
    }
    a.require_size(key + "." + std::to_string(depth * 3) + ".bias", outputs);
    Radial r{};
    r.source = up(a.get<float>(key + ".source"));
    r.target = up(a.get<float>(key + ".target"));
    r.input_t = up(transposed(a.get<float>(key + ".radial"), 64, 10, key + ".radial"));
    r.bias0 = up(a.get<float>(key + ".0.bias"));
    for (int k = 0; k < depth; ++k) {
      std::string base = key + "." + std::to_string(k * 3);
      r.weight_t[k] = k ? up(transposed(a.get<float>(base + ".weight"), 64, 64, base + ".weight")) : nullptr;
      r.bias[k] = up(a.get<float>(base + ".bias"));
      r.gamma[k] = up(a.get<float>(key + "." + std::to_string(k * 3 + 1) + ".weight"));
      r.beta[k] = up(a.get<float>(key + "." + std::to_string(k * 3 + 1) + ".bias"));
    }
    std::string out = key + "." + std::to_string(depth * 3);
    auto ow = a.get<float>(out + ".weight");
    r.out_t = up(transposed(ow, outputs, 64, out + ".weight"));
    if (outputs % 128 == 0)
      r.out = up_split(ow.data(), ow.size());
    r.out_b = up(a.get<float>(out + ".bias"));
    r.depth = depth;
    r.outputs = outputs;
    return r;
  };
  for (int k = 0; k < 2; ++k) {
    auto &l = layers[k];
    std::string p = "layer" + std::to_string(k);
    l.up = get_linear(p + ".linear_up", k ? 2048 : 512, k ? 512 : 128);
    l.res = get_linear(p + ".linear_res", k ? 512 : 128, 9728);
    l.one = get_linear(p + ".linear_1", k ? 5120 : 2048, 9728);
    l.two = get_linear(p + ".linear_2", 8192, 8192);
    l.skip = get_linear(p + ".skip_tp", k ? 2048 : 512, k ? 512 : 2048);
    auto norm = a.get<float>(p + ".norm");
    if (norm.size() < 2)
      throw Error("Invalid MH1 tensor " + p + ".norm");
    l.alpha = norm[0];
    l.beta = norm[1];
    auto dims = a.get<int>(p + ".tp.dims");
    if (dims.size() < 3)
      throw Error("Invalid MH1 tensor " + p + ".tp.dims");
    l.paths = dims[0];
    l.in_comp = dims[1];
    l.out_comp = dims[2];
    if (l.paths != (k ? 10 : 4) || l.in_comp != (k ? 4 : 1) || l.out_comp != (k ? 40 : 16))
      throw Error("Unsupported MH1 tensor product shape");
    auto values = a.get<float>(p + ".tp.values");
    a.require_size(p + ".tp.terms", values.size(), 16);
    auto terms = a.get<TPTerm>(p + ".tp.terms");
    const TPTerm *table = k ? kTP1 : kTP0;
    int table_size = k ? kTPTerms1 : kTPTerms0;
    std::fill(std::begin(l.tp.v), std::end(l.tp.v), 0.f);
    std::vector<bool> seen(table_size, false);
    for (size_t t = 0; t < terms.size(); ++t) {
      auto q = terms[t];
      if (q.path < 0 || q.path >= l.paths || q.in < 0 || q.in >= l.in_comp || q.sh < 0 || q.sh >= 16 ||
          q.out < 0 || q.out >= l.out_comp)
        throw Error("Invalid MH1 tensor-product index");
      int slot = -1;
      for (int s = 0; s < table_size; ++s)
        if (table[s].path == q.path && table[s].in == q.in && table[s].sh == q.sh && table[s].out == q.out)
          slot = s;
      if (slot < 0 || seen[slot])
        throw Error("Unsupported MH1 tensor-product layout: term (" + std::to_string(q.path) + "," +
                    std::to_string(q.in) + "," + std::to_string(q.sh) + "," + std::to_string(q.out) +
                    ") is not in the compiled term table");
      seen[slot] = true;
      l.tp.v[slot] = values[t];
    }
    l.radial = get_radial(p + ".radial", 3, l.paths * 128);
    l.density = get_radial(p + ".density", 1, 1);
    auto poly = a.get<PolyTerm>(p + ".product.terms");
    l.npoly = int(poly.size());
    l.pouts = k ? 1 : 4;
    a.require_size(p + ".product.coefficients", size_t(l.npoly) * 512);
    for (auto t : poly)
      if (t.degree < 1 || t.degree > 3 || t.output < 0 || t.output >= l.pouts || t.a < 0 || t.a >= 16 ||
          (t.degree >= 2 && (t.b < 0 || t.b >= 16)) || (t.degree == 3 && (t.c < 0 || t.c >= 16)))
        throw Error("Invalid MH1 polynomial index");
    {
      auto coef = a.get<float>(p + ".product.coefficients");
      std::vector<int> abc;
      std::vector<float> sorted;
      int starts[4];
      // Per output, terms sorted by (a, b, c) with missing factors as 16 (stable), so the terms
      // sharing a and (a, b) are contiguous.
      for (int o = 0; o < 4; ++o) {
        starts[o] = int(abc.size());
        std::vector<std::pair<int, size_t>> block; // (a | b << 8 | c << 16, term)
        for (size_t t = 0; t < poly.size(); ++t)
          if (poly[t].output == o) {
            const auto &q = poly[t];
            block.push_back({q.a | (q.degree >= 2 ? q.b : 16) << 8 | (q.degree >= 3 ? q.c : 16) << 16, t});
          }
        auto key = [](int v) { return (v & 255) << 16 | ((v >> 8) & 255) << 8 | v >> 16; }; // (a, b, c)
        std::stable_sort(block.begin(), block.end(),
                         [&](const auto &x, const auto &y) { return key(x.first) < key(y.first); });
        for (auto &[packed, t] : block) {
          abc.push_back(packed);
          sorted.insert(sorted.end(), coef.begin() + t * 512, coef.begin() + (t + 1) * 512);
        }
      }
      l.poly_out_start = make_int4(starts[0], starts[1], starts[2], starts[3]);
      // Compiled kernels when the sorted terms are exactly this layer's compiled table.
      auto matches = [&](const PolyABC *table, int count, const int *start, int outputs) {
        if (int(abc.size()) != count || outputs != l.pouts || start[outputs] != count)
          return false;
        for (int o = 0; o < outputs; ++o)
          if (starts[o] != start[o])
            return false;
        for (int t = 0; t < count; ++t)
          if (abc[t] != (table[t].a | table[t].b << 8 | table[t].c << 16))
            return false;
        return true;
      };
      // (MACE_GENERIC_PRODUCT=1 keeps the table-driven kernels for every archive.)
      l.poly_fixed = -1;
      if (!std::getenv("MACE_GENERIC_PRODUCT")) {
        if (k == 0 && matches(kPoly0, kPolyTerms0, kPolyStart0, 4))
          l.poly_fixed = 0;
        else if (k == 1 && matches(kPoly1, kPolyTerms1, kPolyStart1, 1))
          l.poly_fixed = 1;
      }
      l.poly_abc = reinterpret_cast<const int *>(device.upload(abc.data(), abc.size() * 4));
      l.poly_coef_sorted = up(sorted);
    }
    l.plin = get_linear(p + ".product.linear", k ? 512 : 2048, k ? 512 : 2048);
  }
  read0 = get_linear("readout0", 2048, 1);
  read1up = get_linear("readout1.up", 512, 16);
  read1down = get_linear("readout1.down", 16, 1);
}
} // namespace mace
