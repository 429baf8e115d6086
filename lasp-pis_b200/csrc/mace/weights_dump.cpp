// mace-weights-dump MODEL OUTPUT [HEAD]: write the PWMH1001 archive the loader would build
// from MODEL (an MH1 checkpoint, or an archive copied as is).  Host only; same command line
// and exit codes as the reference's mace_weights_dump (mace/tests/weights.cpp:4-16).
#include "checkpoint.hpp"
#include <fstream>
#include <iostream>

int main(int argc, char **argv) {
  try {
    if (argc < 3 || argc > 4)
      throw std::runtime_error("usage: mace-weights-dump MODEL OUTPUT [HEAD]");
    const std::string bytes = mace::weight_data(argv[1], argc == 4 ? argv[3] : "");
    std::ofstream out(argv[2], std::ios::binary);
    if (!out.write(bytes.data(), std::streamsize(bytes.size())))
      throw std::runtime_error("write failed");
  } catch (const std::exception &e) {
    std::cerr << e.what() << "\n";
    return 1;
  }
  return 0;
}
