/* MACE MH1 C ABI of the B200 build.
 *
 * The first six entry points are the reference's ABI with identical signatures and
 * semantics (mace/include/mace/c_api.h:7-15, mace/src/c_api.cpp:18-98): return 0 on
 * success, -1 on failure with a thread-local message from mace_last_error(); create
 * returns NULL on failure; handles are single-flight; outputs are caller-owned, in input
 * atom order, and valid on return; an error does not poison the handle.
 * Backend: 0 Auto, 1 BruteForce, 2 CellList.
 */
#pragma once
#include <mace/export.h>
#include <stddef.h>
#ifdef __cplusplus
extern "C" {
#endif
/* Replaces mace_create_mh1 (mace/include/mace/c_api.h:8). */
MACE_EXPORT void *mace_create_mh1(const char *archive, int backend);
/* Replaces mace_create_mh1_head (mace/include/mace/c_api.h:10).  `model` is a PWMH1001
 * archive or an MH1 PyTorch ZIP checkpoint; a checkpoint is converted for `head` (NULL or ""
 * selects "matpes_r2scan").  Archives carry one head; a non-empty head is rejected for them
 * like the reference does. */
MACE_EXPORT void *mace_create_mh1_head(const char *model, int backend, const char *head);
/* Replaces mace_destroy (mace/include/mace/c_api.h:11). */
MACE_EXPORT void mace_destroy(void *handle);
/* Replaces mace_last_error (mace/include/mace/c_api.h:12); thread-local. */
MACE_EXPORT const char *mace_last_error(void);
/* Replaces mace_calculate (mace/include/mace/c_api.h:13-14).  xyz n x 3 Angstrom, cell
 * 3 x 3 rows, virial 3 x 3 row major = -dE/dstrain (eV).  Null pointers only when n == 0. */
MACE_EXPORT int mace_calculate(void *handle, int n, const float *xyz, const int *elements, const float *cell,
                               double *energy, float *per_atom, float *force, float *virial);
/* Replaces mace_diagnostics (mace/include/mace/c_api.h:15): JSON into buffer. */
MACE_EXPORT int mace_diagnostics(void *handle, char *buffer, size_t capacity);

/* ---- B200 build additions (no counterpart in the reference ABI) ---- */

/* Like mace_create_mh1 but binds the handle to CUDA device `device` (the reference binds
 * to whatever device is current at creation). */
MACE_EXPORT void *mace_create_mh1_device(const char *archive, int backend, int device);
/* Parses and validates a model (PWMH1001 archive, or an MH1 ZIP checkpoint converted for
 * `head`; NULL or "" = "matpes_r2scan") exactly as the constructors do, in host memory: no
 * GPU is needed.  Returns 0, or -1 with the constructor's error in mace_last_error.  No
 * reference counterpart (the reference validates only while creating a handle). */
MACE_EXPORT int mace_check_model(const char *model, const char *head);
/* mace_create_mh1_head bound to CUDA device `device`. */
MACE_EXPORT void *mace_create_mh1_device_head(const char *model, int backend, const char *head, int device);
/* Spatial domain decomposition of one structure across `world` ranks (one process per GPU;
 * B200 build addition, no counterpart in the reference).  Every rank creates its handle with
 * the same 128-byte NCCL id (from mace_nccl_unique_id on one rank) and then calls
 * mace_calculate with the SAME full structure; each rank evaluates the receivers it owns,
 * exchanges layer features, gradients and ghost forces over NCCL, and receives the full
 * result.  Calls on the ranks' handles are collective: every rank must make the same calls
 * in the same order. */
MACE_EXPORT void *mace_create_mh1_domain(const char *archive, int backend, int device, int rank, int world,
                                         const void *nccl_id);
/* Writes a new 128-byte NCCL unique id for mace_create_mh1_domain; returns 0, or -1. */
MACE_EXPORT int mace_nccl_unique_id(void *out128);
/* mace_calculate with DEVICE-resident xyz/elements (device pointers on the handle's GPU);
 * results still land in the caller's host arrays.  Lets a caller that keeps structures in
 * HBM skip the host-to-device copy. */
MACE_EXPORT int mace_calculate_device(void *handle, int n, const float *xyz_device, const int *elements_device,
                                      const float *cell, double *energy, float *per_atom, float *force,
                                      float *virial);
/* Directed edges of the last successful call, in input atom indices: out[5 * k] =
 * (receiver, sender, sx, sy, sz) for k < min(count, capacity), canonically sorted.
 * Returns the edge count (which may exceed capacity) or -1. */
MACE_EXPORT long long mace_last_edges(void *handle, int *out, long long capacity);
/* Turn per-stage device timing on/off for later calls; mace_diagnostics then reports
 * "stages" (name, device ms) and "launches" of the last call.  Returns 0 or -1. */
MACE_EXPORT int mace_profile(void *handle, int enable);
/* Test hook for the node-linear GEMMs: C[z] (+)= A[z] * B on the current device for z < batch,
 * A [batch][M][K], B [K][N], C [batch][M][N] row-major device arrays; mode 0 runs the FP32
 * SIMT kernel, mode 1 the tensor-core (tcgen05, fp16-split) kernel, mode 2 the same as a
 * grouped launch (one problem per batch plane, columns split 128 | N - 128), mode 3 with K
 * split into two segments with their own A and B copies (K >= 64), mode 4 with A given as
 * fp16 split planes and per-64 exponents made on the host (K a multiple of 64).  Blocks;
 * returns 0 or -1.
 * No counterpart in the reference. */
MACE_EXPORT int mace_debug_gemm(int M, int N, int K, int batch, const float *A, const float *B, float *C,
                                int accumulate, int mode);
/* Lapis neighbour list alone (no model): directed edges of a structure at `cutoff` with
 * backend 0/1/2 and an optional grid byte budget (0 = default), in input atom indices,
 * canonically sorted, 5 ints each as in mace_last_edges.  Runs on the current device.
 * Returns the edge count (may exceed capacity) or -1 (message in mace_last_error). */
MACE_EXPORT long long lapis_neighbor_edges(int n, const float *xyz, const float *cell, float cutoff, int backend,
                                           long long grid_bytes, int *out, long long capacity);
/* Neighbour list that allocates no GPU memory.  No counterpart in the reference.
 * For callers that cannot allocate device memory -- hosts that own a fixed device memory pool,
 * run inside another framework's allocator, or forbid allocation during their time step --
 * this builds the same directed edge list as the calculator's neighbour step but keeps all
 * of its scratch in one fixed-size array that the library places in every GPU that loads it
 * (about 512 KiB, held until the process exits).  Inputs are device arrays xyz [n][3] and
 * atomic numbers [n] plus the host cell (3 x 3 rows); outputs are caller-owned device arrays:
 * row [n + 1] (CSR offsets by input atom index), and for each edge the sender, the image
 * shift (3 ints) and the displacement (float4: dx, dy, dz, r; 16-byte aligned).  Candidates
 * are enumerated by brute force over all atoms and periodic images.  Limits: n <= 16384.
 * Returns the edge count E; if E exceeds `capacity` only row is written, so the caller can
 * retry with larger buffers.  Returns -1 on error (message in mace_last_error), including
 * n above the limit.  Runs on the current device and on `stream` (NULL = default stream).
 * The call is synchronous: it waits on `stream` for its results before it returns.  The first
 * call on a device does that device's set-up (it looks up the device address of the array);
 * make that first call before any stream capture.  The set-up is repeated if the device's
 * context is replaced (cudaDeviceReset).  Every call reuses the same array, so calls that
 * overlap on the GPU race with each other: serialise them. */
MACE_EXPORT long long lapis_neighbor_list_static(int n, const float *xyz, const int *elements, const float *cell,
                                                 float cutoff, int *row, int *sender, int *shift, float *vector,
                                                 long long capacity, void *stream);
/* Domain-decomposition exchange plan of one rank, on the current GPU without a communicator
 * (B200 build addition for checks; no counterpart in the reference).  The structure (cutoff
 * Angstrom, all atoms taken as hydrogen) is prepared the way a decomposed evaluation prepares
 * it for rank `rank` of `world`: CSR rows for that rank's receivers only (internal ids
 * [n rank / world, n (rank + 1) / world) of the bin-sorted order).  Outputs: send_counts and
 * ghost_counts [world]; when capacity >= max(E, n) also internal_to_input [n], row
 * [owned + 1], sender [E] (internal ids), ghosts (ascending internal ids) and sends (per peer
 * in rank order, ascending internal ids).  Returns E, the rank's edge count, or -1. */
MACE_EXPORT long long lapis_exchange_plan(int n, const float *xyz, const float *cell, float cutoff, int rank,
                                          int world, int *send_counts, int *ghost_counts, int *internal_to_input,
                                          int *row, int *sender, int *ghosts, int *sends, long long capacity);
/* The same plan from a CSR on the host (no GPU; B200 build addition for checks, no reference
 * counterpart): ids 0..n-1, rank `rank` of `world` owns [n rank / world, n (rank + 1) / world)
 * and gives the rows of those receivers (row [owned + 1], sender ids).  Outputs as above;
 * ghosts and sends are written when capacity >= the larger of their lengths.  Returns 0 or
 * -1 (message in mace_last_error). */
MACE_EXPORT int lapis_exchange_plan_host(int n, int rank, int world, const int *row, const int *sender,
                                         int *send_counts, int *ghost_counts, int *ghosts, int *sends,
                                         long long capacity);
/* Batch of independent periodic cells in one call (B200 build addition; the reference's
 * callers loop over mace_calculate, mace/include/mace/c_api.h:13-14).  Cell c has sizes[c]
 * atoms; xyz (sum(sizes) x 3, Angstrom) and Z (sum(sizes)) are the cells' arrays
 * concatenated in order; cells is count x 9 (lattice vectors as rows).  Outputs are
 * caller-owned: energies[count] (eV), per_atom[sum(sizes)], force[sum(sizes) x 3],
 * virial[count x 9] (row major, -dE/d(strain)).  Per cell the results equal mace_calculate's
 * up to float32 summation order.  Returns 0, or -1 with mace_last_error() set; an error does
 * not poison the handle. */
MACE_EXPORT int mace_calculate_batch(void *handle, int count, const int *sizes, const float *xyz, const int *Z,
                                     const float *cells, double *energies, float *per_atom, float *force,
                                     float *virial);
#ifdef __cplusplus
}
#endif
