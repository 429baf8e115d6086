// Lennard-Jones calculator: the example PairOp of the Lapis extension API (reference:
// lapis/examples/lj/lj.hpp).  Force-shifted potential -- energy and its radial derivative
// vanish at the cutoff; half of each directed edge's energy and virial goes to the receiver,
// together with the full edge force.
#pragma once
#include <lapis/runtime.hpp>

namespace lapis {
class LennardJones final : public Calculator {
  float epsilon_, sigma_;
  Result evaluate() override;

public:
  LennardJones(float epsilon = 1, float sigma = 1, float cutoff = 2.5, Options options = {});
};
} // namespace lapis
