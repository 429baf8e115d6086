// Symbol visibility for the MACE C ABI (the reference generates this header from CMake's
// GenerateExportHeader; mace/CMakeLists.txt:39).
#pragma once
#ifndef MACE_EXPORT
#define MACE_EXPORT __attribute__((visibility("default")))
#endif
