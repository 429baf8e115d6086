/* C entry point for the Lapis Lennard-Jones example (B200 build addition; the reference
 * exposes LennardJones only through C++, lapis/examples/lj/lj.hpp).  Same input and output
 * conventions as mace_calculate (mace/include/mace/c_api.h): xyz n x 3 in Angstrom, lattice
 * vectors as rows, outputs in input order; returns 0, or -1 with mace_last_error() set. */
#ifndef LAPIS_LJ_H
#define LAPIS_LJ_H
#include <mace/export.h>
#ifdef __cplusplus
extern "C" {
#endif
MACE_EXPORT int lapis_lj_calculate(int n, const float *xyz, const int *Z, const float *cell, float epsilon,
                                   float sigma, float cutoff, int backend, double *energy, float *per_atom,
                                   float *force, float *virial);
#ifdef __cplusplus
}
#endif
#endif
