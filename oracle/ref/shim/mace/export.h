/* Stand-in for the export header the reference's CMake generates
 * (mace/CMakeLists.txt:39, GenerateExportHeader): default visibility for the C ABI. */
#pragma once
#define MACE_EXPORT __attribute__((visibility("default")))
