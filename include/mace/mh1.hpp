// mace::MH1 -- the C++ model API (same surface as mace/include/mace/mh1.hpp:6-19).
#pragma once
#include <lapis/domain.hpp>
#include <lapis/runtime.hpp>
#include <mace/export.h>
#include <memory>
namespace mace {
class MACE_EXPORT MH1 final : public lapis::Calculator {
  struct Model;
  std::unique_ptr<Model> model_;
  std::vector<lapis::Result> compute(bool batch); // the evaluation; one result or one per cell
  lapis::Result evaluate() override;
  std::vector<lapis::Result> evaluate_batch() override;

public:
  // `model` is a PWMH1001 archive or an MH1 PyTorch ZIP checkpoint, which is converted on
  // the host for `head` ("matpes_r2scan" when empty).  An empty head is required for
  // archives (they carry one head).
  explicit MH1(const std::string &model, lapis::Options options = {});
  MH1(const std::string &model, lapis::Options options, const std::string &head);
  ~MH1() override;
  size_t parameter_bytes() const;
  // Per-stage CUDA-event timing of each call into diagnostics().stages (also enabled by the
  // MACE_PROFILE_MH1 environment variable, which additionally prints them to stderr).
  void set_profiling(bool enabled);
  lapis::Result calculate_file(const std::string &path, size_t frame = 0);
  // Evaluate structures decomposed across ranks (B200 build addition): every rank passes the
  // same full structure and gets the full result; null returns to single-GPU evaluation.
  void set_domain(std::shared_ptr<lapis::Domain> domain);
};
} // namespace mace
