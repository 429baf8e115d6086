// Kernel launch helper: every launch of this library goes through it so that the number
// of kernels a call issues is counted (Diagnostics::launches, reported by bench.py).
#pragma once
#include "lapis/runtime.hpp"
#include <utility>

namespace lapis {
template <class... KernelArgs, class... Args>
inline void launch(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   Args &&...args) {
  kernel<<<grid, block, smem, stream>>>(std::forward<Args>(args)...);
  ++launch_counter();
}
} // namespace lapis
