// MH1 parameter layout on the device and the kernel entry points of the B200 build.
//
// Node tensors use the reference's [irrep block][component][node][channel] layout
// (mace/src/mh1.cu:83-84): every equivariant linear is then, per path and component, a
// row-major GEMM with nodes as rows.  Edge tensors are indexed by the CSR edge id of the
// Lapis runtime (receiver-major).
#pragma once
#include "lapis/runtime.hpp"
#include "tp_table.h"
#include <cuda.h>
#include <string>
#include <vector>

namespace mace {

struct LinearPath {
  int in_offset, out_offset, in_mul, out_mul, dim, weight_offset;
};
// Operand B of the tensor-core GEMM: a K-major matrix [N][K] split as B 2^exp = hi + lo,
// two fp16 planes (split_f16).
struct TCMatrix {
  const uint16_t *hi = nullptr, *lo = nullptr;
  int exp = 0;
  explicit operator bool() const { return hi != nullptr; }
};
// An fp32 array written as the tensor-core GEMM's split operand: element i is
// (hi[i] + lo[i]) 2^-exp[i / 64], hi and lo fp16 (bit patterns) rounded to nearest, with one
// exponent per 64 consecutive elements (a row's K slab) that brings the slab's largest
// magnitude into [2^14, 2^15) (split_exponent).  The GEMM then loads both planes by TMA and
// skips its own split.
struct SplitPlanes {
  uint16_t *hi = nullptr, *lo = nullptr;
  int16_t *exp = nullptr;
  explicit operator bool() const { return hi != nullptr; }
};
// Tensor-core copies of one path's weight W [in_mul][out_mul]: forward planes are K-major for
// Y = X W ([out_mul][in_mul]), backward planes for X_grad = Y_grad W^T ([in_mul][out_mul]).
// Empty when the shape is not eligible.
struct TCWeights {
  TCMatrix fwd, bwd;
};
struct Linear {
  int input = 0, output = 0;
  std::vector<LinearPath> paths;
  std::vector<TCWeights> tc;     // per path
  const float *weight = nullptr; // device, [in_mul][out_mul] per path
};
// Radial MLP weights, transposed at load for coalesced per-unit access.
struct Radial {
  const float *source, *target; // [species][64]
  const float *input_t;         // [10][64]
  const float *bias0;           // [64]
  const float *weight_t[3];     // [64 in][64 out]; entry 0 unused
  const float *bias[3], *gamma[3], *beta[3];
  const float *out_t;           // [64][outputs]
  const float *out_b;           // [outputs]
  TCMatrix out;                 // [outputs][64] fp16 split of the projection (tensor cores)
  int depth, outputs;
};
struct PolyTerm {
  int output, degree, a, b, c;
};
struct TPValues {
  float v[128]; // coupling values in the compiled term order (tp_table.h)
};
struct Layer {
  Linear up, res, one, two, skip, plin;
  Radial radial, density;
  float alpha, beta;
  TPValues tp;
  // Terms sorted by output (stable): factor indices a | b << 8 | c << 16 with missing
  // factors = 16 (a constant 1), coefficient rows in the same order, and the first term of
  // each output (entries past `pouts` equal npoly).
  const int *poly_abc;
  const float *poly_coef_sorted;
  int4 poly_out_start;
  // Which compiled product table (product_table.h) the sorted terms equal, or -1 (generic
  // table-driven kernels).
  int poly_fixed = -1;
  int npoly, pouts, paths, in_comp, out_comp;
};

struct Device {
  std::vector<void *> allocations;
  // Validation without a GPU: uploads are copied into host memory instead.
  bool host_only = false;
  ~Device();
  float *upload(const void *data, size_t bytes);
};

struct ModelData {
  Device device;
  Layer layers[2];
  Linear read0, read1up, read1down;
  float constants[14];
  const float *constants_dev, *embedding, *bessel, *radii, *zbl_radii, *zbl_c;
  const int *lookup;  // [119] atomic number -> species index or -1
  const float *e0_z;  // [119] baseline energy by atomic number
  size_t bytes = 0;
  int species = 0;
  // `path` is a PWMH1001 archive (head must be empty) or an MH1 ZIP checkpoint, converted
  // for `head` ("matpes_r2scan" when empty).
  void load(const std::string &path, const std::string &head = {});
  // Every parse and validation step of load() with host memory in place of the device, so
  // a model can be checked where no GPU is present.
  void validate(const std::string &path, const std::string &head = {});
};

// ---- kernels (edge_kernels.cu / node_kernels.cu) ----
struct EdgeArrays {
  float *basis, *dbasis; // [E][10]
  float2 *cut;           // [E] (cut, dcut)
  float *Y;              // [E][16]
  float *dY;             // [E][16][3] dY/dd (written when non-null)
};
struct RadialOut {
  float *h, *dh;        // [E][64]
  float2 *density;      // [E] (value, d/dr)
};

void launch_species(cudaStream_t, const lapis::DeviceGeometry &, const int *lookup, int *species);
void launch_embed(cudaStream_t, int n, const int *species, const float *embedding, float *x);
void launch_zbl(cudaStream_t, const lapis::DeviceGeometry &, const float *constants, const float *radii,
                const float *coeff, float shift, float *energy, float *force, float *virial);
// pair[e] = sender species | receiver species << 16 (written by launch_edge_geometry).
void launch_edge_geometry(cudaStream_t, const lapis::DeviceGeometry &, const int *species, const float *constants,
                          const float *radii, const float *bessel, EdgeArrays, int *pair);
// Radial and density MLPs of `count` (at most two) layers in one launch, a grid row per
// layer, into ro[k].  scaled: ro.h / ro.dh receive cut h and cut dh + dcut h (for the
// projection path, whose GEMMs then produce cut h W and its r-derivative cut dh W + dcut h W).
void launch_radial(cudaStream_t, const lapis::DeviceGeometry &, const Layer *const *layers, const RadialOut *ro,
                   int count, const int *pair, EdgeArrays, bool scaled = false);
void launch_message_forward(cudaStream_t, int layer, const lapis::DeviceGeometry &, const Layer &, EdgeArrays,
                            RadialOut, const float *up, float *message, float *density);
// ug_edge (layer 1): each edge's up-projection gradient, [E][4][128]; summed onto the senders
// by launch_sender_gather.
void launch_message_backward(cudaStream_t, int layer, const lapis::DeviceGeometry &, const Layer &,
                             EdgeArrays, RadialOut, const float *up, const float *message_grad,
                             const float *density_grad, float *ug_edge, float4 *edge_force, bool accumulate);
// Projection path (edge_proj.cu): the radial projection R = h W (and dR = dh W) runs as a
// tensor-core GEMM into a buffer covering the edges of receivers [r0, r1) = [e0, e1); the
// tensor-product kernels read rows e - e0.
struct ProjectionChunk {
  int r0, r1;
  long long e0, e1;
};
// n_up: row stride of up / up_grad (senders; 0: the receiver count g.n).  message_split set:
// the messages go out as SplitPlanes (the tensor-core linear_1's input) instead of fp32.
void launch_message_forward_proj(cudaStream_t, int layer, const lapis::DeviceGeometry &, const Layer &, EdgeArrays,
                                 RadialOut, const ProjectionChunk &, const float *R, const float *up,
                                 float *message, float *density, int n_up = 0, SplitPlanes message_split = {});
// ug_edge (layer 1): the chunk's per-edge up-projection gradients, row e - e0 of [rows][4][128].
void launch_message_backward_proj(cudaStream_t, int layer, const lapis::DeviceGeometry &, const Layer &,
                                  EdgeArrays, RadialOut, const ProjectionChunk &, const float *R, const float *dR,
                                  const float *up, const float *message_grad, const float *density_grad,
                                  float *ug_edge, float4 *edge_force, bool accumulate, int n_up = 0);
// Edges per projection chunk (bounds the R / dR buffers at 2 x 1280 floats per edge):
// 2^20, or MACE_PROJECTION_CHUNK_EDGES when set to a positive value.
long long projection_chunk_edges();
void launch_force_gather(cudaStream_t, const lapis::DeviceGeometry &, const float4 *edge_force, float *force,
                         float *virial);
// Domain-decomposed form: reverse edges outside the local graph (index < 0) are skipped; the
// reactions on ghost senders come from launch_ghost_reactions.
void launch_force_gather_domain(cudaStream_t, const lapis::DeviceGeometry &, const float4 *edge_force, float *force,
                                float *virial);

// Sender index (sender_gather.cu): for each sender j < n, its edges in ascending edge order,
// edges[offsets[j] .. offsets[j + 1]).  Sender-side sums run over it in that order, so they
// are bitwise reproducible (no float atomics).
struct SenderIndex {
  int n;
  int *offsets, *edges;
};
SenderIndex build_sender_index(cudaStream_t, lapis::Context &, long long E, int n_senders, const int *sender);
// out[q][j][c] (row stride `stride`) += sum over sender j's edges e in [e0, e1) of
// rows[e - e0][q][c], for q < comps (4) and 128 channels c.
void launch_sender_gather(cudaStream_t, const SenderIndex &, long long e0, long long e1, const float *rows, int comps,
                          float *out, int stride);
// force[j] -= sum of the edge forces of ghost sender j, for j in [n_own, index.n).
void launch_ghost_reactions(cudaStream_t, const SenderIndex &, int n_own, const float4 *edge_force, float *force);

// Equivariant linear over n nodes: Y (+)= X W per path and component, or the transposed
// product for the backward.  Paths with tensor-core-eligible shapes run on tc_gemm.
// nx / ny: row stride of x's / y's component blocks (0: n), for arrays with rows beyond the n
// computed ones (the ghost rows of a domain-decomposed evaluation).
// xs: x given as SplitPlanes (every path on the tensor cores, input widths multiples of 64).
void linear(cudaStream_t, int n, const Linear &, const float *x, float *y, bool backward = false,
            bool add = false, int *status = nullptr, int nx = 0, int ny = 0, const SplitPlanes *xs = nullptr);
// Whether linear() can take its input as SplitPlanes (tensor-core linears, every path eligible).
bool linear_takes_split(const Linear &, bool backward);
// Tensor-core GEMM (tc_gemm.cu): C[z] (+)= A[z] B, B given as its fp16 split, K-major [N][K].
bool tc_gemm_supported(int N, int K);
void tc_gemm(cudaStream_t, int M, int N, int K, int batch, const float *A, long long strideA, const TCMatrix &B,
             float *C, int ldc, long long strideC, bool accumulate, int *status);
// A group of independent tensor-core GEMMs in one persistent launch (per 16 problems).  A
// spec with `join` set is a further K segment of the previous spec's problem (same C, M, N,
// batch and mode; its own A, K and B): C (+)= sum over the segments of A_s B_s.
struct GemmSpec {
  int M, N, K, batch;
  const float *A;
  long long strideA;
  TCMatrix B;
  float *C;
  int ldc;
  long long strideC;
  bool accumulate;
  bool join = false;
  // A given already split (SplitPlanes, K a multiple of 64): its planes at A's element
  // offset (batch stride strideA), its exponents (one per row and 64-wide slab, batch stride
  // strideAexp); A itself is then not read.
  const uint16_t *Ahi = nullptr, *Alo = nullptr;
  const int16_t *Aexp = nullptr;
  long long strideAexp = 0;
};
void tc_gemm_group(cudaStream_t, const GemmSpec *specs, int count, int *status);
// Host split of a weight matrix: w 2^exp = hi + lo, both fp16 (bit patterns) rounded to
// nearest, with exp such that the largest |w| 2^exp lies in [2^14, 2^15).  Returns exp.
int split_f16(const float *w, size_t count, uint16_t *hi, uint16_t *lo);
// Use the tensor-core path in linear() (default true; MACE_SIMT_LINEARS=1 disables).
bool tensor_core_linears();
// Edge kernels over tensor-core radial projections (default true; false with SIMT linears or
// MACE_SIMT_EDGES=1, which selects the fused SIMT edge kernels).
bool projection_edges();
// pre = raw / (alpha + beta density) + res is not stored: the backward recomputes it from raw
// and res (the same FP32 expression, so the same values).  pre_grad may alias res.
// gs set: the gate goes out as SplitPlanes (the tensor-core linear_2's input) instead of fp32.
void launch_normalize_gate(cudaStream_t, int n, const float *raw, const float *res, const float *density,
                           float alpha, float beta, float scalar_scale, float gate_scale, float *gate,
                           SplitPlanes gs = {});
// raw_grad_split set: raw_grad goes out as SplitPlanes (the tensor-core linear_1 backward's input).
void launch_gate_norm_backward(cudaStream_t, int n, const float *res, const float *raw, const float *density,
                               const float *gate_grad, float alpha, float beta, float scalar_scale,
                               float gate_scale, float *pre_grad, float *raw_grad, float *density_grad,
                               SplitPlanes raw_grad_split = {});
void launch_product(cudaStream_t, int n, const Layer &, const float *x, float *y);
// xgs set (compiled MH1 tables only): the input gradient goes out as SplitPlanes (the
// tensor-core linear_2 backward's input) instead of fp32.
void launch_product_backward(cudaStream_t, int n, const Layer &, const float *x, const float *grad, float *xg,
                             SplitPlanes xgs = {});
void launch_add(cudaStream_t, size_t count, const float *a, float *b, float scale);
void launch_fill(cudaStream_t, size_t count, float *a, float value);
void launch_readout_act(cudaStream_t, int count, const float *x, const float *grad, float *y, float scale,
                        bool backward);
} // namespace mace
