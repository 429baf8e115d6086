// BIOSYM/LASP .arc structure reader (the format chemio/src/arc.cpp:35-93 parses): frames
// of "PBC a b c alpha beta gamma" + "El x y z CORE ..." lines closed by a double "end".
#pragma once
#include <array>
#include <cstddef>
#include <string>
#include <vector>

namespace mace {
struct ArcFrame {
  std::vector<double> positions; // Cartesian Angstrom, n x 3
  std::vector<int> elements;
  std::array<double, 9> cell{};  // lattice vectors are rows
  std::array<bool, 3> pbc{false, false, false};
  std::string title;
};
// Lattice rows from lengths and angles (degrees): a along x, b in the xy plane.
std::array<double, 9> cell_from_parameters(double a, double b, double c, double alpha, double beta, double gamma);
std::vector<ArcFrame> read_arc(const std::string &path);
ArcFrame read_arc_frame(const std::string &path, std::size_t frame = 0);
} // namespace mace
