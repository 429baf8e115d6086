// mace-main: command-line front end of the B200 MH1 engine.
//
// Contract (the reference CLI's, mace/src/main.cpp:12-133):
//   mace-main MODEL STRUCTURE.arc [--frame N] [--backend auto|brute|cell] [--head NAME]
//             [--json] [--output FILE]
//   exit 0 on success, 1 on any error (message on stderr), 2 when MODEL or STRUCTURE is
//   missing (usage on stdout); `--help` alone prints the usage and exits 0.  The model's head
//   is announced on stderr.  Results go to stdout or to FILE, which may not name an input.
//
// This implementation parses the command line into a Request through a table of option
// handlers, evaluates it with mace::MH1::calculate_file, renders the whole report into one
// string (floats with 9 significant digits, which round-trip float32 exactly; the float64
// energy with 17) and writes it in one piece.
#include <cstdio>
#include <filesystem>
#include <fstream>
#include <functional>
#include <iostream>
#include <mace/mh1.hpp>
#include <map>
#include <stdexcept>
#include <string>

namespace {
constexpr const char *kUsage = "Usage: mace-main MODEL STRUCTURE.arc [--frame N] [--backend auto|brute|cell] "
                               "[--head NAME] [--json] [--output FILE]\n";

struct Request {
  std::string model, structure, head, output;
  size_t frame = 0;
  bool json = false;
  lapis::Options options;
};

size_t parse_frame(const std::string &text) {
  bool digits = !text.empty();
  for (char ch : text)
    digits = digits && ch >= '0' && ch <= '9';
  if (!digits)
    throw std::runtime_error("frame must be a nonnegative integer");
  return size_t(std::stoull(text));
}

lapis::NeighborBackend parse_backend(const std::string &text) {
  static const std::map<std::string, lapis::NeighborBackend> names = {
      {"auto", lapis::NeighborBackend::Auto},
      {"brute", lapis::NeighborBackend::BruteForce},
      {"cell", lapis::NeighborBackend::CellList}};
  auto it = names.find(text);
  if (it == names.end())
    throw std::runtime_error("unknown backend: " + text);
  return it->second;
}

// Options after the two positional arguments.  Flags with a value consume the next word.
Request parse(int argc, char **argv) {
  Request r;
  r.model = argv[1];
  r.structure = argv[2];
  using Setter = std::function<void(Request &, const std::string &)>;
  const std::map<std::string, Setter> valued = {
      {"--frame", [](Request &q, const std::string &v) { q.frame = parse_frame(v); }},
      {"--backend", [](Request &q, const std::string &v) { q.options.backend = parse_backend(v); }},
      {"--head", [](Request &q, const std::string &v) { q.head = v; }},
      {"--output", [](Request &q, const std::string &v) { q.output = v; }}};
  for (int k = 3; k < argc; ++k) {
    std::string word = argv[k];
    if (word == "--json") {
      r.json = true;
      continue;
    }
    auto it = valued.find(word);
    if (it == valued.end())
      throw std::runtime_error("unknown option: " + word);
    if (k + 1 >= argc)
      throw std::runtime_error("missing value for " + word);
    it->second(r, argv[++k]);
  }
  return r;
}

// An existing output path may not be the model or the structure file (same inode).
void check_output_path(const Request &r) {
  namespace fs = std::filesystem;
  if (r.output.empty() || !fs::exists(r.output))
    return;
  for (const std::string *input : {&r.model, &r.structure})
    if (fs::equivalent(r.output, *input))
      throw std::runtime_error("output would overwrite an input file");
}

// A ZIP checkpoint starts with "PK"; the converter picks a head from it.  An archive
// carries exactly one head.
std::string head_banner(const Request &r) {
  std::ifstream in(r.model, std::ios::binary);
  char magic[2] = {0, 0};
  bool zip = in.read(magic, 2) && magic[0] == 'P' && magic[1] == 'K';
  if (!zip)
    return "fixed by processed archive";
  return r.head.empty() ? "matpes_r2scan" : r.head;
}

std::string number(double v, int digits) {
  char buf[40];
  std::snprintf(buf, sizeof buf, "%.*g", digits, v);
  return buf;
}

std::string render(const Request &r, const lapis::Result &res) {
  const size_t atoms = res.energies.size();
  auto f32 = [](float v) { return number(v, 9); };
  std::string s;
  if (r.json) {
    s += "{\"frame\":" + std::to_string(r.frame) + ",\"atoms\":" + std::to_string(atoms);
    s += ",\"units\":{\"energy\":\"eV\",\"forces\":\"eV/Angstrom\",\"virial\":\"eV\"}";
    s += ",\"energy\":" + number(res.energy, 17) + ",\"atomic_energies\":[";
    for (size_t i = 0; i < atoms; ++i)
      s += (i ? "," : "") + f32(res.energies[i]);
    s += "],\"forces\":[";
    for (size_t i = 0; i < atoms; ++i)
      s += std::string(i ? ",[" : "[") + f32(res.forces[3 * i]) + "," + f32(res.forces[3 * i + 1]) + "," +
           f32(res.forces[3 * i + 2]) + "]";
    s += "],\"virial\":[";
    for (int k = 0; k < 9; ++k)
      s += (k ? "," : "") + f32(res.virial[k]);
    s += "]}\n";
    return s;
  }
  s += "Frame: " + std::to_string(r.frame) + "\nAtoms: " + std::to_string(atoms) +
       "\nEnergy (eV): " + number(res.energy, 17) + "\nForces (eV/Angstrom), input atom order:\n";
  for (size_t i = 0; i < atoms; ++i)
    s += std::to_string(i) + " " + f32(res.forces[3 * i]) + " " + f32(res.forces[3 * i + 1]) + " " +
         f32(res.forces[3 * i + 2]) + "\n";
  s += "Virial (eV), -dE/dstrain, row major:\n";
  for (int row = 0; row < 3; ++row)
    s += f32(res.virial[3 * row]) + " " + f32(res.virial[3 * row + 1]) + " " + f32(res.virial[3 * row + 2]) + "\n";
  return s;
}

void emit(const Request &r, const std::string &text) {
  if (r.output.empty()) {
    std::cout << text << std::flush;
    if (!std::cout)
      throw std::runtime_error("failed to write inference output");
    return;
  }
  std::ofstream file(r.output, std::ios::binary | std::ios::trunc);
  if (!file)
    throw std::runtime_error("cannot open output: " + r.output);
  file << text;
  file.flush();
  if (!file)
    throw std::runtime_error("failed to write inference output");
}
} // namespace

int main(int argc, char **argv) {
  if (argc == 2 && std::string(argv[1]) == "--help") {
    std::cout << kUsage;
    return 0;
  }
  if (argc < 3) {
    std::cout << kUsage;
    return 2;
  }
  try {
    Request r = parse(argc, argv);
    check_output_path(r);
    mace::MH1 model(r.model, r.options, r.head);
    lapis::Result result = model.calculate_file(r.structure, r.frame);
    std::cerr << "MACE head: " << head_banner(r) << "\n";
    emit(r, render(r, result));
    return 0;
  } catch (const std::exception &e) {
    std::cerr << "mace-main: " << e.what() << '\n';
    return 1;
  }
}
