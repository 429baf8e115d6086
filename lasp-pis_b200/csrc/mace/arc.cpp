// .arc reader.  Same accepted syntax and error conditions as the reference's Chemio parser
// (chemio/src/arc.cpp:23-93): "!" comment lines, PBC=ON / PBC=OFF headers outside frames,
// a title line, an optional PBC cell record before the atoms, atom lines whose fifth field
// is CORE, and two "end" markers closing every frame; errors carry path:line.
#include "arc.hpp"
#include <algorithm>
#include <cctype>
#include <cmath>
#include <fstream>
#include <iterator>
#include <sstream>
#include <stdexcept>
#include <unordered_map>

namespace mace {
namespace {
const char *const kSymbols =
    "H He Li Be B C N O F Ne Na Mg Al Si P S Cl Ar K Ca Sc Ti V Cr Mn Fe Co Ni Cu Zn Ga Ge As Se Br Kr Rb Sr Y "
    "Zr Nb Mo Tc Ru Rh Pd Ag Cd In Sn Sb Te I Xe Cs Ba La Ce Pr Nd Pm Sm Eu Gd Tb Dy Ho Er Tm Yb Lu Hf Ta W Re "
    "Os Ir Pt Au Hg Tl Pb Bi Po At Rn Fr Ra Ac Th Pa U Np Pu Am Cm Bk Cf Es Fm Md No Lr Rf Db Sg Bh Hs Mt Ds Rg "
    "Cn Nh Fl Mc Lv Ts Og";

int atomic_number(const std::string &symbol) {
  static const std::unordered_map<std::string, int> table = [] {
    std::unordered_map<std::string, int> t;
    std::istringstream in(kSymbols);
    std::string s;
    for (int z = 1; in >> s; ++z)
      t.emplace(s, z);
    return t;
  }();
  auto it = table.find(symbol);
  return it == table.end() ? 0 : it->second;
}

// The whitespace operator>> skips in the C locale.
bool blank(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\v' || c == '\f' || c == '\r'; }

// Whitespace-separated fields of one line, reusing the strings' storage between lines.
struct Fields {
  std::vector<std::string> word;
  size_t count = 0;
  void split(const std::string &line) {
    count = 0;
    for (size_t i = 0, n = line.size();;) {
      while (i < n && blank(line[i]))
        ++i;
      if (i == n)
        return;
      size_t j = i;
      while (j < n && !blank(line[j]))
        ++j;
      if (count == word.size())
        word.emplace_back();
      word[count++].assign(line, i, j - i);
      i = j;
    }
  }
  const std::string &operator[](size_t k) const { return word[k]; }
  size_t size() const { return count; }
  bool empty() const { return count == 0; }
};

double parse_number(const std::string &s) {
  std::size_t used = 0;
  double x = std::stod(s, &used);
  if (used != s.size() || !std::isfinite(x))
    throw std::runtime_error("invalid number: " + s);
  return x;
}
} // namespace

std::array<double, 9> cell_from_parameters(double a, double b, double c, double alpha, double beta, double gamma) {
  for (double x : {a, b, c, alpha, beta, gamma})
    if (!std::isfinite(x) || x <= 0)
      throw std::runtime_error("invalid cell parameters");
  if (alpha >= 180 || beta >= 180 || gamma >= 180)
    throw std::runtime_error("invalid cell angles");
  const double deg = 3.14159265358979323846 / 180;
  double ca = std::cos(alpha * deg), cb = std::cos(beta * deg), cg = std::cos(gamma * deg),
         sg = std::sin(gamma * deg);
  double cx = c * cb, cy = c * (ca - cb * cg) / sg, cz2 = c * c - cx * cx - cy * cy;
  if (sg < 1e-12 || cz2 <= c * c * 1e-14)
    throw std::runtime_error("degenerate or impossible cell");
  return {a, 0, 0, b * cg, b * sg, 0, cx, cy, std::sqrt(cz2)};
}

std::vector<ArcFrame> read_arc(const std::string &path) {
  auto dot = path.find_last_of('.');
  std::string ext = dot == std::string::npos ? "" : path.substr(dot);
  std::transform(ext.begin(), ext.end(), ext.begin(), [](unsigned char ch) { return char(std::tolower(ch)); });
  if (ext != ".arc")
    throw std::runtime_error("unsupported structure format: " + ext + " (supported: .arc)");
  std::ifstream in(path, std::ios::binary);
  if (!in)
    throw std::runtime_error("cannot open structure: " + path);
  // The whole file at once, then '\n'-separated lines as getline would return them.
  const std::string text((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
  if (in.bad())
    throw std::runtime_error("error reading structure: " + path);
  std::vector<ArcFrame> frames;
  ArcFrame cur;
  bool periodic = false, have_cell = false, first_end = false, pending = false;
  std::string line;
  Fields f;
  std::size_t lineno = 0;
  for (size_t at = 0; at < text.size();) {
    const size_t eol = std::min(text.find('\n', at), text.size());
    line.assign(text, at, eol - at);
    at = eol + 1;
    ++lineno;
    try {
      f.split(line);
      if (f.empty() || f[0][0] == '!')
        continue;
      if (f[0] == "PBC=ON" || f[0] == "PBC=OFF") {
        if (pending || have_cell)
          throw std::runtime_error("periodicity header inside frame");
        periodic = f[0] == "PBC=ON";
        continue;
      }
      if (f[0] == "end" || f[0] == "END") {
        if (cur.elements.empty())
          throw std::runtime_error("empty frame");
        if (!first_end) {
          first_end = true;
          continue;
        }
        cur.pbc = {periodic, periodic, periodic};
        if (periodic && !have_cell)
          throw std::runtime_error("periodic frame has no cell");
        frames.push_back(std::move(cur));
        cur = ArcFrame{};
        have_cell = first_end = pending = false;
        continue;
      }
      if (first_end)
        throw std::runtime_error("expected second end marker");
      if (f[0] == "PBC") {
        if (have_cell || !cur.elements.empty() || f.size() < 7)
          throw std::runtime_error("invalid PBC record");
        cur.cell = cell_from_parameters(parse_number(f[1]), parse_number(f[2]), parse_number(f[3]),
                                        parse_number(f[4]), parse_number(f[5]), parse_number(f[6]));
        have_cell = pending = true;
        continue;
      }
      if (f.size() >= 5 && f[4] == "CORE") {
        if (periodic && !have_cell)
          throw std::runtime_error("atom before cell");
        int z = atomic_number(f[0]);
        if (!z)
          throw std::runtime_error("unknown element: " + f[0]);
        cur.elements.push_back(z);
        for (int k = 1; k <= 3; ++k)
          cur.positions.push_back(parse_number(f[k]));
        pending = true;
        continue;
      }
      if (have_cell || !cur.elements.empty())
        throw std::runtime_error("unrecognized atom record");
      if (pending)
        throw std::runtime_error("unexpected frame title");
      cur.title = line;
      pending = true;
    } catch (const std::exception &e) {
      throw std::runtime_error(path + ":" + std::to_string(lineno) + ": " + e.what());
    }
  }
  if (pending || have_cell || first_end)
    throw std::runtime_error(path + ": incomplete ARC frame");
  if (frames.empty())
    throw std::runtime_error(path + ": no structures");
  return frames;
}

ArcFrame read_arc_frame(const std::string &path, std::size_t frame) {
  auto frames = read_arc(path);
  if (frame >= frames.size())
    throw std::runtime_error("frame index out of range: " + std::to_string(frame));
  return std::move(frames[frame]);
}
} // namespace mace
