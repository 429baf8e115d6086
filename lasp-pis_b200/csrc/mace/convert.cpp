// MH1 checkpoint -> PWMH1001 archive conversion (host only).
//
// Input: a PyTorch ZIP checkpoint of a six-head, two-layer ScaleShiftMACE (MACE MH1).
// Output: the archive records the loader reads, for one head.  The record set, the checks
// and the arithmetic follow mace/src/weights.cpp:305-393 so that both produce the same bytes:
//
// * tensors are widened to double, combined in double and rounded to float32 once;
// * e3nn path weights are folded into every linear and embedding (weights.cpp:94-140);
// * the radial MLP's 1034-wide first layer is split into a 10-wide radial part and per-species
//   source/target rows, the species embeddings contracted in double in ascending input order
//   (weights.cpp:156-192);
// * tensor-product values are float32(coupling) * float32(path weight) (weights.cpp:200-240);
// * the symmetric contraction's coupling tensors U are symmetrised over the distinct
//   permutations of each sorted index tuple, in lexicographic order, and contracted with the
//   per-channel weights (weights.cpp:241-303).
//
// The file is compiled without floating-point contraction, so each product and sum is
// rounded exactly where the reference rounds it.
#include "cg_table.h"
#include "checkpoint.hpp"
#include <algorithm>
#include <cmath>
#include <cstring>
#include <fstream>
#include <map>
#include <numeric>
#include <stdexcept>

namespace mace {
namespace {

using ckpt::Node;
using ckpt::NodeRef;

[[noreturn]] void reject(const std::string &what) {
  throw std::runtime_error("unsupported MH1 checkpoint: " + what);
}
void need(bool ok, const std::string &what) {
  if (!ok)
    reject(what);
}

ckpt::Tensor tensor_of(const NodeRef &m, const std::string &path) {
  NodeRef v = ckpt::walk(m, path);
  need(v->kind == Node::TensorView, "expected tensor " + path);
  return v->tensor;
}
std::vector<double> values_of(const NodeRef &m, const std::string &path) { return tensor_of(m, path).values(); }
// A Python number or a one-element tensor.  Anything else fails as a tensor without
// storage would ("checkpoint: invalid tensor metadata"), as in the reference.
double scalar_of(const NodeRef &m, const std::string &path) {
  NodeRef v = ckpt::walk(m, path);
  if (v->kind == Node::Number)
    return v->number;
  auto d = v->kind == Node::TensorView ? v->tensor.values() : ckpt::Tensor{}.values();
  need(d.size() == 1, "expected scalar " + path);
  return d[0];
}
size_t child_count(const NodeRef &m, const std::string &path) {
  return ckpt::walk(m, path)->field("_modules")->fields.size();
}

// One (mul, l, parity) block of an e3nn Irreps, with its offset in the flattened feature
// vector and its first component index (sum of 2l+1 over earlier blocks).
struct Block {
  int mul, l, parity, offset, component;
  int dim() const { return 2 * l + 1; }
};
std::vector<Block> irreps_of(const NodeRef &node) {
  need(node->items.size() <= 64, "too many irreps");
  std::vector<Block> out;
  int offset = 0, component = 0;
  for (NodeRef x : node->items) {
    // _MulIr pickles as Cls((mul, ir)): unwrap the single argument tuple.
    if (x->items.size() == 1)
      x = x->item(0);
    const int64_t mul = x->item(0)->integer();
    const NodeRef &ir = x->item(1);
    const int64_t l = ir->item(0)->integer(), parity = ir->item(1)->integer();
    need(mul > 0 && mul <= 4096 && l >= 0 && l <= 3 && (parity == 1 || parity == -1), "irreps");
    out.push_back({int(mul), int(l), int(parity), offset, component});
    offset += int(mul) * (2 * int(l) + 1);
    component += 2 * int(l) + 1;
  }
  need(!out.empty(), "empty irreps");
  return out;
}
int width_of(const std::vector<Block> &r) { return r.back().offset + r.back().mul * r.back().dim(); }

// The archive under construction: records sorted by name, as the archive lists them.
class Records {
public:
  void floats(const std::string &name, const std::vector<double> &v) {
    std::string bytes(v.size() * 4, '\0');
    bool finite = true;
    for (size_t i = 0; i < v.size(); ++i) {
      const float f = float(v[i]);
      finite = finite && std::isfinite(v[i]) && std::isfinite(f);
      std::memcpy(&bytes[i * 4], &f, 4);
    }
    need(finite, "nonfinite " + name);
    add(name, std::move(bytes));
  }
  void ints(const std::string &name, const std::vector<int> &v) {
    std::string bytes(v.size() * 4, '\0');
    for (size_t i = 0; i < v.size(); ++i) {
      const int32_t x = v[i];
      std::memcpy(&bytes[i * 4], &x, 4);
    }
    add(name, std::move(bytes));
  }
  std::string encode() const {
    size_t total = 12;
    for (const auto &[name, data] : records_)
      total += 12 + name.size() + data.size();
    std::string out;
    out.reserve(total);
    out += "PWMH1001";
    append<uint32_t>(out, uint32_t(records_.size()));
    for (const auto &[name, data] : records_) {
      append<uint32_t>(out, uint32_t(name.size()));
      append<uint64_t>(out, uint64_t(data.size()));
      out += name;
      out += data;
    }
    return out;
  }

private:
  std::map<std::string, std::string> records_;
  void add(const std::string &name, std::string bytes) {
    need(records_.emplace(name, std::move(bytes)).second, "duplicate " + name);
  }
  template <class T> static void append(std::string &s, T x) {
    char b[sizeof(T)];
    std::memcpy(b, &x, sizeof(T));
    s.append(b, sizeof(T));
  }
};

std::vector<int> iota_list(int n, int start = 0) {
  std::vector<int> v(static_cast<size_t>(n));
  std::iota(v.begin(), v.end(), start);
  return v;
}

// An e3nn o3.Linear: one [in_mul][out_mul] block per instruction, scaled by its path weight.
// `rows` / `cols` pick input / output channels (head selection of the readouts), which is
// only defined for single-block irreps.
void emit_linear(Records &ar, const std::string &name, const NodeRef &m, const std::vector<int> &rows = {},
                 const std::vector<int> &cols = {}) {
  const auto ins = irreps_of(ckpt::walk(m, "irreps_in")), outs = irreps_of(ckpt::walk(m, "irreps_out"));
  const auto w = values_of(m, "weight");
  const NodeRef instructions = ckpt::walk(m, "instructions");
  need(instructions->items.size() <= 128, "linear path count");
  std::vector<int> paths;
  std::vector<double> packed;
  size_t consumed = 0;
  for (const NodeRef &inst : instructions->items) {
    const int64_t i = inst->item(0)->integer(), o = inst->item(1)->integer();
    need(i >= 0 && i < int64_t(ins.size()) && o >= 0 && o < int64_t(outs.size()), "linear instruction indices");
    const Block &bi = ins[size_t(i)], &bo = outs[size_t(o)];
    need(bi.l == bo.l && bi.parity == bo.parity, "linear irreps mismatch");
    const NodeRef &shape = inst->item(2);
    need(shape->items.size() == 2 && shape->item(0)->integer() == bi.mul && shape->item(1)->integer() == bo.mul,
         "linear path shape");
    const size_t block = size_t(bi.mul) * size_t(bo.mul);
    need(consumed + block <= w.size(), "linear weight count");
    if (!rows.empty())
      need(ins.size() == 1, "input head selection");
    if (!cols.empty())
      need(outs.size() == 1, "output head selection");
    const std::vector<int> r = rows.empty() ? iota_list(bi.mul) : rows;
    const std::vector<int> c = cols.empty() ? iota_list(bo.mul) : cols;
    paths.insert(paths.end(), {rows.empty() ? bi.offset : 0, cols.empty() ? bo.offset : 0, int(r.size()),
                               int(c.size()), bi.dim(), int(packed.size())});
    const double path_weight = inst->item(3)->number;
    for (int a : r)
      need(a >= 0 && a < bi.mul, "head index");
    for (int b : c)
      need(b >= 0 && b < bo.mul, "head index");
    packed.reserve(packed.size() + r.size() * c.size());
    for (int a : r) {
      const double *row = &w[consumed + size_t(a) * size_t(bo.mul)];
      for (int b : c)
        packed.push_back(row[b] * path_weight);
    }
    consumed += block;
  }
  need(consumed == w.size(), "unconsumed linear weights");
  ar.ints(name + ".paths", paths);
  ar.ints(name + ".dims", {rows.empty() ? width_of(ins) : int(rows.size()),
                           cols.empty() ? width_of(outs) : int(cols.size())});
  ar.floats(name + ".weight", packed);
}

// A species one-hot -> 512x0e e3nn Linear, with its path weight folded in.
std::vector<double> species_embedding(const NodeRef &m, int species) {
  const auto ins = irreps_of(ckpt::walk(m, "irreps_in")), outs = irreps_of(ckpt::walk(m, "irreps_out"));
  const NodeRef instructions = ckpt::walk(m, "instructions");
  need(ins.size() == 1 && outs.size() == 1 && ins[0].l == 0 && outs[0].l == 0 && ins[0].mul == species &&
           outs[0].mul == 512 && instructions->items.size() == 1,
       "embedding architecture");
  auto w = values_of(m, "weight");
  need(w.size() == size_t(species) * 512, "embedding weights");
  const NodeRef &inst = instructions->item(0);
  need(inst->item(0)->integer() == 0 && inst->item(1)->integer() == 0, "embedding path");
  const double path_weight = inst->item(3)->number;
  for (double &x : w)
    x *= path_weight;
  return w;
}

// MACE's radial MLP: net = [Linear(1034, 64), LayerNorm, SiLU] * depth + [Linear(64, out)].
// The first layer's input is [10 radial features | source embedding | target embedding].
void emit_radial(Records &ar, const std::string &name, const NodeRef &m, const std::vector<double> &source,
                 const std::vector<double> &target, int species, int depth, int outputs) {
  const NodeRef net = ckpt::walk(m, "net");
  const auto w = values_of(net, "0.weight");
  need(tensor_of(net, "0.weight").shape == std::vector<int64_t>{64, 1034}, "radial input dimensions");
  std::vector<double> s(size_t(species) * 64), t(size_t(species) * 64), r(64 * 10);
  for (int z = 0; z < species; ++z)
    for (int o = 0; o < 64; ++o) {
      const double *src = &source[size_t(z) * 512], *tgt = &target[size_t(z) * 512];
      const double *ws = &w[size_t(o) * 1034 + 10], *wt = &w[size_t(o) * 1034 + 522];
      double as = 0, at = 0;
      for (int i = 0; i < 512; ++i) {
        as += src[i] * ws[i];
        at += tgt[i] * wt[i];
      }
      s[size_t(z) * 64 + o] = as;
      t[size_t(z) * 64 + o] = at;
    }
  for (int o = 0; o < 64; ++o)
    for (int i = 0; i < 10; ++i)
      r[size_t(o) * 10 + i] = w[size_t(o) * 1034 + i];
  ar.floats(name + ".source", s);
  ar.floats(name + ".target", t);
  ar.floats(name + ".radial", r);
  need(net->field("_modules")->fields.size() == size_t(depth) * 3 + 1, "radial network depth");
  for (int k = 0; k <= depth * 3; ++k) {
    const std::string key = std::to_string(k);
    const NodeRef layer = ckpt::walk(net, key);
    if (k % 3 == 2) {
      need(layer->text == "torch.nn.modules.activation SiLU", "radial activation");
      continue;
    }
    if (k % 3 == 1)
      need(scalar_of(layer, "eps") == 1e-5, "radial LayerNorm epsilon");
    else
      need(tensor_of(layer, "weight").shape ==
               std::vector<int64_t>{k == depth * 3 ? outputs : 64, k == 0 ? 1034 : 64},
           "radial matrix shape");
    ar.floats(name + "." + key + ".weight", values_of(layer, "weight"));
    ar.floats(name + "." + key + ".bias", values_of(layer, "bias"));
  }
}

// The channel-wise ("uvu") e3nn TensorProduct of node features with the l <= 3 harmonics.
void emit_tensor_product(Records &ar, const std::string &name, const NodeRef &m, int layer) {
  const auto ins = irreps_of(ckpt::walk(m, "irreps_in1")), sh = irreps_of(ckpt::walk(m, "irreps_in2")),
             outs = irreps_of(ckpt::walk(m, "irreps_out"));
  const NodeRef instructions = ckpt::walk(m, "instructions");
  need(instructions->items.size() == size_t(layer ? 10 : 4), "tensor product path count");
  need(sh.size() == 4, "spherical harmonic irreps");
  for (int l = 0; l < 4; ++l)
    need(sh[size_t(l)].l == l && sh[size_t(l)].mul == 1 && sh[size_t(l)].parity == (l % 2 ? -1 : 1),
         "spherical harmonic convention");
  std::vector<int> terms;
  std::vector<double> values;
  int path = 0;
  for (const NodeRef &inst : instructions->items) {
    const int64_t i = inst->item(0)->integer(), j = inst->item(1)->integer(), o = inst->item(2)->integer();
    need(i >= 0 && i < int64_t(ins.size()) && j >= 0 && j < int64_t(sh.size()) && o >= 0 &&
             o < int64_t(outs.size()),
         "tensor product instruction");
    const NodeRef &shape = inst->item(6);
    need(inst->item(3)->text == "uvu" && inst->item(4)->integer() == 1 && shape->items.size() == 2 &&
             shape->item(0)->integer() == 128 && shape->item(1)->integer() == 1,
         "tensor product connectivity");
    const Block &bi = ins[size_t(i)], &bs = sh[size_t(j)], &bo = outs[size_t(o)];
    need(bi.l <= 1 && bi.mul == 128 && bo.mul == 128, "tensor product multiplicity");
    const float path_weight = float(inst->item(5)->number);
    bool any = false;
    for (const Coupling &cg : kCouplingTable)
      if (cg.l1 == bi.l && cg.l2 == bs.l && cg.lo == bo.l) {
        any = true;
        terms.insert(terms.end(), {path, bi.component + cg.a, bs.l * bs.l + cg.b, bo.component + cg.c});
        values.push_back(double(cg.value * path_weight));
      }
    need(any, "unavailable coupling coefficients");
    ++path;
  }
  ar.ints(name + ".terms", terms);
  ar.floats(name + ".values", values);
  ar.ints(name + ".dims", {path, ins.back().component + ins.back().dim(), outs.back().component + outs.back().dim()});
}

// MACE's SymmetricContraction (correlation 3) as sparse symmetric monomials: for every output
// component and sorted index tuple a <= b <= c over the 16 feature components, the per-channel
// coefficient sum_p (sum over distinct permutations of U[out, perm, p]) * w[p, channel].
void emit_polynomial(Records &ar, const std::string &name, const NodeRef &product, int layer) {
  const int contractions = layer ? 1 : 2;
  need(child_count(product, "symmetric_contractions.contractions") == size_t(contractions),
       "product contraction count");
  std::vector<int> terms;
  std::vector<double> coefficients;
  int out_offset = 0;
  for (int c = 0; c < contractions; ++c) {
    const NodeRef con = ckpt::walk(product, "symmetric_contractions.contractions." + std::to_string(c));
    need(scalar_of(con, "correlation") == 3, "product correlation");
    const int outputs = c == 0 ? 1 : 3;
    for (int degree = 1; degree <= 3; ++degree) {
      const ckpt::Tensor ut = tensor_of(con, "U_matrix_" + std::to_string(degree));
      const auto u = ut.values();
      const ckpt::Tensor wt = tensor_of(con, degree == 3 ? "weights_max" : "weights." + std::to_string(2 - degree));
      const auto w = wt.values();
      need(wt.shape.size() == 3 && wt.shape[0] == 1 && wt.shape[2] == 512, "contraction weight shape");
      const int64_t paths = wt.shape[1];
      std::vector<int64_t> expected;
      if (outputs > 1)
        expected.push_back(outputs);
      expected.insert(expected.end(), size_t(degree), 16);
      expected.push_back(paths);
      need(ut.shape == expected, "coupling tensor shape");
      std::vector<double> coupling(static_cast<size_t>(paths)), coeff(512);
      for (int out = 0; out < outputs; ++out)
        for (int a = 0; a < 16; ++a)
          for (int b = degree >= 2 ? a : 0; b < (degree >= 2 ? 16 : 1); ++b)
            for (int d = degree == 3 ? b : 0; d < (degree == 3 ? 16 : 1); ++d) {
              int idx[3] = {a, b, d};
              std::fill(coupling.begin(), coupling.end(), 0.0);
              std::fill(coeff.begin(), coeff.end(), 0.0);
              do {
                size_t flat = size_t(out);
                for (int k = 0; k < degree; ++k)
                  flat = flat * 16 + size_t(idx[k]);
                const double *row = &u[flat * size_t(paths)];
                for (int64_t p = 0; p < paths; ++p)
                  coupling[size_t(p)] += row[p];
              } while (std::next_permutation(idx, idx + degree));
              for (int64_t p = 0; p < paths; ++p) {
                const double k = coupling[size_t(p)];
                if (k == 0)
                  continue;
                const double *wp = &w[size_t(p) * 512];
                for (int ch = 0; ch < 512; ++ch)
                  coeff[size_t(ch)] += k * wp[ch];
              }
              double largest = 0;
              for (double x : coeff)
                largest = std::max(largest, std::fabs(x));
              if (largest < 1e-12)
                continue;
              terms.insert(terms.end(), {out_offset + out, degree, a, degree >= 2 ? b : -1, degree == 3 ? d : -1});
              coefficients.insert(coefficients.end(), coeff.begin(), coeff.end());
            }
    }
    out_offset += outputs;
  }
  ar.ints(name + ".terms", terms);
  ar.floats(name + ".coefficients", coefficients);
}

std::string convert(const ckpt::Zip &zip, const std::string &requested) {
  const NodeRef root = ckpt::load(zip);
  need(root->text == "mace.modules.models ScaleShiftMACE", "expected ScaleShiftMACE");
  const NodeRef heads = ckpt::walk(root, "heads");
  const std::string head_name = requested.empty() ? "matpes_r2scan" : requested;
  int head = -1;
  for (size_t i = 0; i < heads->items.size(); ++i)
    if (heads->item(i)->text == head_name)
      head = int(i);
  need(head >= 0, "unknown head: " + head_name);
  need(heads->items.size() == 6, "expected six-head MH1 architecture");
  need(child_count(root, "interactions") == 2 && child_count(root, "products") == 2 &&
           child_count(root, "readouts") == 2,
       "two-layer architecture");
  need(scalar_of(root, "r_max") == 6 && scalar_of(root, "radial_embedding.apply_cutoff") == 0, "radial cutoff");

  Records ar;
  const auto numbers = values_of(root, "atomic_numbers");
  const int species = int(numbers.size());
  need(species > 0 && species <= 118, "element count");
  std::vector<int> z;
  for (double x : numbers) {
    need(x == std::trunc(x) && x >= 1 && x <= 118, "atomic number");
    z.push_back(int(x));
  }
  ar.ints("atomic_numbers", z);
  ar.floats("embedding", species_embedding(ckpt::walk(root, "node_embedding.linear"), species));
  const auto e0 = values_of(root, "atomic_energies_fn.atomic_energies");
  need(e0.size() == heads->items.size() * size_t(species), "atomic baseline shape");
  ar.floats("e0", std::vector<double>(e0.begin() + std::ptrdiff_t(head) * species,
                                      e0.begin() + std::ptrdiff_t(head + 1) * species));
  const auto scales = values_of(root, "scale_shift.scale"), shifts = values_of(root, "scale_shift.shift");
  need(scales.size() == 6 && shifts.size() == 6, "scale-shift shape");

  const NodeRef re = ckpt::walk(root, "radial_embedding"), zbl = ckpt::walk(root, "pair_repulsion_fn");
  const std::string gate = "interactions.0.equivariant_nonlin.";
  ar.floats("constants", {6, scalar_of(re, "bessel_fn.prefactor"), scalar_of(re, "cutoff_fn.p"),
                          scalar_of(re, "distance_transform.a"), scalar_of(re, "distance_transform.q"),
                          scalar_of(re, "distance_transform.p"), scales[size_t(head)], shifts[size_t(head)],
                          scalar_of(zbl, "a_exp"), scalar_of(zbl, "a_prefactor"), scalar_of(zbl, "p"),
                          scalar_of(root, gate + "act_scalars.acts.0.cst"),
                          scalar_of(root, gate + "act_gates.acts.0.cst"),
                          scalar_of(root, "readouts.1.non_linearity.acts.0.cst")});
  for (const char *act : {"act_scalars", "act_gates"})
    need(scalar_of(root, gate + act + ".acts.0.cst") ==
             scalar_of(root, std::string("interactions.1.equivariant_nonlin.") + act + ".acts.0.cst"),
         "different gate normalization");
  ar.floats("bessel", values_of(re, "bessel_fn.bessel_weights"));
  ar.floats("radii", values_of(re, "distance_transform.covalent_radii"));
  ar.floats("zbl.radii", values_of(zbl, "covalent_radii"));
  ar.floats("zbl.c", values_of(zbl, "c"));

  for (int layer = 0; layer < 2; ++layer) {
    const std::string prefix = "layer" + std::to_string(layer);
    const NodeRef block = ckpt::walk(root, "interactions." + std::to_string(layer));
    need(block->text == "mace.modules.blocks RealAgnosticResidualNonLinearInteractionBlock", "interaction class");
    for (const char *lin : {"linear_up", "linear_res", "linear_1", "linear_2", "skip_tp"})
      emit_linear(ar, prefix + "." + lin, ckpt::walk(block, lin));
    ar.floats(prefix + ".norm", {scalar_of(block, "alpha"), scalar_of(block, "beta")});
    const auto source = species_embedding(ckpt::walk(block, "source_embedding"), species);
    const auto target = species_embedding(ckpt::walk(block, "target_embedding"), species);
    emit_radial(ar, prefix + ".radial", ckpt::walk(block, "conv_tp_weights"), source, target, species, 3,
                (layer ? 10 : 4) * 128);
    emit_radial(ar, prefix + ".density", ckpt::walk(block, "density_fn"), source, target, species, 1, 1);
    emit_tensor_product(ar, prefix + ".tp", ckpt::walk(block, "conv_tp"), layer);
    const NodeRef product = ckpt::walk(root, "products." + std::to_string(layer));
    emit_polynomial(ar, prefix + ".product", product, layer);
    emit_linear(ar, prefix + ".product.linear", ckpt::walk(product, "linear"));
  }
  emit_linear(ar, "readout0", ckpt::walk(root, "readouts.0.linear"), {}, {head});
  const auto lanes = iota_list(16, head * 16);
  emit_linear(ar, "readout1.up", ckpt::walk(root, "readouts.1.linear_1"), {}, lanes);
  emit_linear(ar, "readout1.down", ckpt::walk(root, "readouts.1.linear_2"), lanes, {head});
  return ar.encode();
}

} // namespace

std::string convert_checkpoint(std::vector<char> zip_bytes, const std::string &head) {
  return convert(ckpt::Zip(std::move(zip_bytes)), head);
}

std::string weight_data(const std::string &path, const std::string &head) {
  if (ckpt::is_zip(path))
    return convert(ckpt::Zip(path), head);
  need(head.empty(), "head selection requires an original checkpoint; an archive already contains one head");
  std::ifstream in(path, std::ios::binary | std::ios::ate);
  const auto size = in.tellg();
  need(size >= 0 && uint64_t(size) < (uint64_t(1) << 31), "archive size");
  std::string bytes(size_t(size), '\0');
  in.seekg(0);
  if (!in.read(bytes.data(), std::streamsize(bytes.size())))
    throw std::runtime_error("cannot read MH1 archive: " + path);
  return bytes;
}

} // namespace mace
