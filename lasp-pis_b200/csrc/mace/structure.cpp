// MH1::calculate_file: evaluates one frame of an ARC trajectory (the reference's
// mace/src/structure.cpp:7-31 contract: three periodic axes are required, coordinates and
// the cell must be representable in float32, results are in input atom order).
//
// The ARC reader returns float64 positions and a float64 cell; the engine takes float32.
// Each value is narrowed once, and a value that overflows float32 (or was not finite) is an
// error naming the array it came from.
#include "arc.hpp"
#include "mace/mh1.hpp"
#include <climits>
#include <cmath>

namespace mace {
namespace {
template <class Out> void narrow(const double *in, size_t count, Out *out, const char *what) {
  for (size_t k = 0; k < count; ++k) {
    float v = static_cast<float>(in[k]);
    if (!std::isfinite(v))
      throw lapis::Error(std::string(what) + " exceeds float32 range");
    out[k] = v;
  }
}
} // namespace

lapis::Result MH1::calculate_file(const std::string &path, size_t frame) {
  ArcFrame f = read_arc_frame(path, frame);
  for (bool periodic : f.pbc)
    if (!periodic)
      throw lapis::Error("mace requires three periodic axes");
  const size_t atoms = f.elements.size();
  if (atoms > size_t(INT_MAX))
    throw lapis::Error("too many atoms");
  std::vector<float> xyz(f.positions.size());
  narrow(f.positions.data(), f.positions.size(), xyz.data(), "coordinate");
  lapis::Structure s;
  narrow(f.cell.data(), 9, s.cell.data(), "cell");
  s.size = int(atoms);
  s.positions = xyz.data();
  s.elements = f.elements.data();
  s.pbc = f.pbc;
  return calculate(s);
}
} // namespace mace
