// mace-host-bench: times this build's host-side I/O, the CPU work a caller pays before any
// device call.
//
//   mace-host-bench arc FILE [REPEAT]        read_arc_frame(FILE, 0)
//   mace-host-bench convert MODEL [REPEAT]   weight_data(MODEL, ""): checkpoint conversion,
//                                            or the archive read for a PWMH1001 file
//   mace-host-bench arc-dump FILE FRAME      the parsed frame as JSON (parity tests)
//
// Prints one JSON object with the median and minimum wall time over REPEAT runs (default 20)
// after one untimed run.  Single-threaded, like the reference's code for these steps
// (chemio/src/arc.cpp, mace/src/weights.cpp).
#include "arc.hpp"
#include "checkpoint.hpp"
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <stdexcept>
#include <string>
#include <vector>

int main(int argc, char **argv) {
  try {
    if (argc < 3 || argc > 4)
      throw std::runtime_error("usage: mace-host-bench arc|convert FILE [REPEAT] | arc-dump FILE FRAME");
    const std::string what = argv[1], file = argv[2];
    if (what == "arc-dump") {
      const auto frame = std::size_t(std::atol(argc == 4 ? argv[3] : "0"));
      const auto s = mace::read_arc_frame(file, frame);
      std::printf("{\"title\": \"");
      for (unsigned char c : s.title)
        if (c == '"' || c == '\\')
          std::printf("\\%c", c);
        else if (c < 0x20)
          std::printf("\\u%04x", c);
        else
          std::putchar(c);
      std::printf("\", \"pbc\": [%d, %d, %d], \"cell\": [", int(s.pbc[0]), int(s.pbc[1]), int(s.pbc[2]));
      for (int k = 0; k < 9; ++k)
        std::printf("%s%.17g", k ? ", " : "", s.cell[size_t(k)]);
      std::printf("], \"elements\": [");
      for (size_t k = 0; k < s.elements.size(); ++k)
        std::printf("%s%d", k ? ", " : "", s.elements[k]);
      std::printf("], \"positions\": [");
      for (size_t k = 0; k < s.positions.size(); ++k)
        std::printf("%s%.17g", k ? ", " : "", s.positions[k]);
      std::printf("]}\n");
      return 0;
    }
    const int repeat = argc == 4 ? std::atoi(argv[3]) : 20;
    if (repeat < 1)
      throw std::runtime_error("REPEAT must be positive");
    size_t units = 0;
    std::function<void()> run;
    if (what == "arc")
      run = [&] { units = mace::read_arc_frame(file, 0).elements.size(); };
    else if (what == "convert")
      run = [&] { units = mace::weight_data(file, "").size(); };
    else
      throw std::runtime_error("unknown step " + what);
    run();
    std::vector<double> ms;
    for (int k = 0; k < repeat; ++k) {
      const auto t = std::chrono::steady_clock::now();
      run();
      ms.push_back(std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t).count());
    }
    std::sort(ms.begin(), ms.end());
    const double median = repeat % 2 ? ms[repeat / 2] : 0.5 * (ms[repeat / 2 - 1] + ms[repeat / 2]);
    std::printf("{\"step\": \"%s\", \"units\": %zu, \"median_ms\": %.3f, \"min_ms\": %.3f, \"repeat\": %d}\n",
                what.c_str(), units, median, ms[0], repeat);
  } catch (const std::exception &e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 1;
  }
  return 0;
}
