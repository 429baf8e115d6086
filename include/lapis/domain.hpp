// Spatial domain decomposition of one periodic structure across ranks (one process per GPU),
// B200 build addition for large structures (no counterpart in the reference, whose
// calculators evaluate a structure on one GPU).
//
// Every rank passes the same full structure.  partition() makes the context build CSR rows
// only for the receivers this rank owns -- a contiguous range of the bin-sorted internal
// order, i.e. a compact slab -- so each rank enumerates and stores its own edges only.
// localize() then switches the context to this rank's graph: the owned receivers and, as
// senders, those plus the ghost atoms their edges reach, numbered after them.  The
// evaluation exchanges only what crosses ranks, point to point over NCCL on the context's
// stream: layer features of ghost senders (owners -> ghosts), their gradients and the ghost
// sender forces (ghosts -> owners), and finally the per-atom outputs (an all-reduce of the
// owned rows), so every rank returns the full result.  NCCL is loaded at run time
// (libnccl.so.2, the copy already in the process when there is one).
//
// Failures: the communicator is non-blocking; every NCCL step and every wait for the
// exchanges has a deadline (MACE_DOMAIN_TIMEOUT_S seconds, default 120).  A peer that never
// takes part, an asynchronous NCCL error, or ranks whose structures or exchange plans
// disagree (checked by an all-gather before any point-to-point step) make the call throw on
// the ranks that see it; a timed-out or failed communicator is aborted and the domain stays
// failed (later calls throw at once).
#pragma once
#include "runtime.hpp"
#include <memory>
#include <string>

namespace lapis {
// A new NCCL unique id (128 bytes) for Domain's communicator; made by one rank, passed to all.
std::string nccl_unique_id();

class Domain {
public:
  Domain(int rank, int world, const void *unique_id);
  ~Domain();
  Domain(const Domain &) = delete;
  Domain &operator=(const Domain &) = delete;
  int rank() const;
  int world() const;
  // Owned receivers n_own = rows [0, n_own); senders n_local = owned then ghosts.
  int n_own() const;
  int n_local() const;
  // Sets ctx.part / ctx.parts so that Context::prepare builds this rank's rows only.
  void partition(Context &ctx) const;
  // After ctx.prepare (partitioned): ctx.geometry becomes the local graph.
  void localize(Context &ctx);
  // Back to the full geometry (for Context::finish).
  void restore(Context &ctx);
  // Rows [n_own, n_local) of x ([comps][stride][width] floats) from their owners.  Runs on the
  // domain's own stream after the work enqueued so far on ctx.stream; call join() before
  // ctx.stream reads the ghost rows (work that does not read them may run meanwhile).
  void fetch_ghost_rows(Context &ctx, float *x, int comps, int stride, int width);
  // Adds rows [n_own, n_local) of x into the owners' rows (ghosts -> owners); asynchronous
  // like fetch_ghost_rows: join() before ctx.stream reads the owned rows of x.
  void return_ghost_rows(Context &ctx, float *x, int comps, int stride, int width);
  // ctx.stream waits for the exchanges issued so far.
  void join(Context &ctx);
  // Owned rows of e [n_own], f [n_own][3], v [n_own][9] into full-structure arrays (internal
  // order), summed over ranks so every rank holds all atoms.  ef, ff, vf must be one contiguous
  // buffer: ff = ef + n, vf = ef + 4 n (n = full atom count).
  void gather_outputs(Context &ctx, const float *e, const float *f, const float *v, float *ef, float *ff, float *vf);

private:
  struct Impl;
  std::unique_ptr<Impl> impl_;
};
} // namespace lapis
