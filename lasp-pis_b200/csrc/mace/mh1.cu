// mace::MH1 for B200: model construction and the forward + analytical backward evaluation.
//
// Stage order and scaling follow the reference's MH1::evaluate (mace/src/mh1.cu:754-898):
// embedding and ZBL, two interaction layers (up/res/skip linears, messages + density,
// linear_1, density normalisation, gate, linear_2, symmetric contraction, product linear +
// skip, layer-0 readout), the SiLU readout of layer 1, then the reverse pass (readout VJPs,
// product / gate / normalisation VJPs, linear transposes, edge backward for layers 1 and 0).
// Energies are scale (constants[6]) x readouts + shift (constants[7]) + ZBL; the per-element
// baseline e0 is added in float64 for the total (mace/src/mh1.cu:890-896).
#include "mace/mh1.hpp"
#include "model.hpp"
#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstdio>
#include <cstring>

namespace mace {
using namespace lapis;

// Replay of a recorded evaluation.  A single-structure call whose prepared geometry is
// byte-for-byte the previous call's (atom and edge counts, cell, every workspace pointer) and
// whose workspaces did not grow enqueues exactly the same kernels with the same arguments:
// the second such call is captured into a CUDA graph, and later ones launch that graph
// instead of ~70 kernels one by one.  Positions live in device buffers the graph reads, so a
// replay evaluates the current coordinates; any change of the key (n, E, cell, buffers)
// drops back to launching kernels directly.  Not used for batches, decomposed handles,
// profiling, or more than one projection chunk (their host-side steps cannot be captured).
struct GraphKey {
  lapis::DeviceGeometry geometry;
  size_t allocated = 0;
  bool valid = false;
  bool matches(const lapis::Context &c) const {
    return valid && allocated == c.diagnostics.allocated_bytes &&
           std::memcmp(&geometry, &c.geometry, sizeof geometry) == 0;
  }
  void set(const lapis::Context &c) {
    std::memcpy(&geometry, &c.geometry, sizeof geometry);
    allocated = c.diagnostics.allocated_bytes;
    valid = true;
  }
};
struct GraphCache {
  GraphKey seen;      // the last direct (eager) call's key
  GraphKey recorded;  // the key of exec
  cudaGraphExec_t exec = nullptr;
  float *energy = nullptr, *force = nullptr, *virial = nullptr;
  int launches = 0;
  void drop() {
    if (exec)
      cudaGraphExecDestroy(exec);
    exec = nullptr;
    recorded.valid = false;
  }
  ~GraphCache() { drop(); }
};

bool graphs_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("MACE_CUDA_GRAPHS");
    return !(v && v[0] == '0');
  }();
  return on;
}

struct MH1::Model {
  ModelData data;
  bool profiling = false;
  std::shared_ptr<lapis::Domain> domain;
  std::vector<cudaEvent_t> events;
  GraphCache graph;
  ~Model() {
    for (auto e : events)
      cudaEventDestroy(e);
  }
};

MH1::MH1(const std::string &archive, Options o, const std::string &head)
    : Calculator(6, o), model_(std::make_unique<Model>()) {
  model_->data.load(archive, head);
}
MH1::MH1(const std::string &archive, Options o) : MH1(archive, o, {}) {}
MH1::~MH1() = default;
size_t MH1::parameter_bytes() const { return model_->data.bytes; }
void MH1::set_profiling(bool enabled) { model_->profiling = enabled; }
void MH1::set_domain(std::shared_ptr<lapis::Domain> domain) {
  model_->domain = std::move(domain);
  if (model_->domain)
    model_->domain->partition(context_);
  else
    context_.part = 0, context_.parts = 1;
}

long long projection_chunk_edges() {
  static const long long edges = [] {
    const char *v = std::getenv("MACE_PROJECTION_CHUNK_EDGES");
    long long k = v ? std::atoll(v) : 0;
    return k > 0 ? k : 1ll << 20;
  }();
  return edges;
}

namespace {
// Receiver-aligned chunks of at most projection_chunk_edges() edges (a receiver with more
// edges gets a chunk of its own) for the projection path; a single chunk, without a host
// copy of the CSR offsets, when all edges fit.
std::vector<ProjectionChunk> projection_chunks(Context &c) {
  int n = c.geometry.n;
  long long E = c.geometry.edge_capacity, cap = projection_chunk_edges();
  if (E <= cap)
    return {ProjectionChunk{0, n, 0, E}};
  std::vector<int> row(size_t(n) + 1);
  check(cudaMemcpyAsync(row.data(), c.geometry.edge_offsets, row.size() * sizeof(int), cudaMemcpyDeviceToHost,
                        c.stream));
  check(cudaStreamSynchronize(c.stream));
  std::vector<ProjectionChunk> chunks;
  for (int r = 0; r < n;) {
    int r1 = r + 1;
    while (r1 < n && row[r1 + 1] - row[r] <= cap)
      ++r1;
    chunks.push_back(ProjectionChunk{r, r1, row[r], row[r1]});
    r = r1;
  }
  return chunks;
}

// Per-stage timing (like the reference's StageTimer, mace/src/mh1.cu:53-82): CUDA events
// recorded on the model stream between stages, taken from a persistent pool so that the
// timed path creates no events.
struct StageTimer {
  cudaStream_t stream;
  bool enabled, print;
  std::vector<cudaEvent_t> &pool;
  std::vector<std::string> names;
  StageTimer(cudaStream_t s, bool on, std::vector<cudaEvent_t> &events)
      : stream(s), enabled(on || std::getenv("MACE_PROFILE_MH1")), print(std::getenv("MACE_PROFILE_MH1")),
        pool(events) {
    mark("start");
  }
  void mark(const std::string &name) {
    if (!enabled)
      return;
    if (names.size() == pool.size()) {
      cudaEvent_t e;
      check(cudaEventCreate(&e));
      pool.push_back(e);
    }
    check(cudaEventRecord(pool[names.size()], stream));
    names.push_back(name);
  }
  // Intervals between consecutive marks, summed per name (chunked stages mark once per chunk).
  void report(Diagnostics &d) {
    d.stages.clear();
    if (!enabled || names.size() < 2)
      return;
    check(cudaEventSynchronize(pool[names.size() - 1]));
    for (size_t k = 1; k < names.size(); ++k) {
      float ms = 0;
      check(cudaEventElapsedTime(&ms, pool[k - 1], pool[k]));
      auto it = std::find_if(d.stages.begin(), d.stages.end(), [&](const auto &x) { return x.first == names[k]; });
      if (it == d.stages.end())
        d.stages.emplace_back(names[k], ms);
      else
        it->second += ms;
    }
    if (print)
      for (auto &x : d.stages)
        std::fprintf(stderr, "MH1 %s: %.4f ms\n", x.first.c_str(), x.second);
  }
};
} // namespace

Result MH1::evaluate() { return compute(false)[0]; }
std::vector<Result> MH1::evaluate_batch() { return compute(true); }

std::vector<Result> MH1::compute(bool batch) {
  auto &c = context_;
  auto &m = model_->data;
  cudaStream_t s = c.stream;
  lapis::Domain *dom = model_->domain.get();
  if (dom && batch)
    throw Error("Batched calls do not combine with domain decomposition");
  int n_full = c.geometry.n;
  if (n_full > INT_MAX / 9728)
    throw Error("MH1 node dimensions exceed v1 int32 capacity");
  StageTimer timer(s, model_->profiling, model_->events);
  GraphCache &gc = model_->graph;
  bool replayable = graphs_enabled() && !batch && !dom && !timer.enabled &&
                    c.geometry.edge_capacity <= projection_chunk_edges();
  float *energy = nullptr, *force = nullptr, *virial = nullptr;
  auto finish = [&]() {
    timer.mark("finish-enqueue");
    std::vector<Result> results;
    if (batch)
      results = c.finish_batch(energy, force, virial, m.e0_z);
    else
      results.push_back(c.finish(energy, force, virial, m.e0_z));
    timer.report(c.diagnostics);
    return results;
  };
  c.diagnostics.graph = "direct";
  if (replayable && gc.exec && gc.recorded.matches(c)) {
    c.diagnostics.graph = "replayed";
    check(cudaGraphLaunch(gc.exec, s));
    energy = gc.energy, force = gc.force, virial = gc.virial;
    launch_counter() += gc.launches;
    auto results = finish();
    c.diagnostics.launches = launch_counter();
    return results;
  }
  // The second call with the same key is recorded (the first one sized every workspace).
  bool record = replayable && gc.seen.matches(c);
  if (replayable)
    gc.seen.set(c);
  else
    gc.seen.valid = false;
  int launches_before = launch_counter();
  auto enqueue = [&]() {
  // Domain decomposition: the context switches to this rank's graph -- owned receivers
  // (rows [0, n)) and, for the sender-indexed arrays, ghost rows [n, ns) after them.
  if (dom)
    dom->localize(c);
  struct Restore {
    lapis::Domain *d;
    Context &c;
    ~Restore() {
      if (d)
        d->restore(c);
    }
  } restore_geometry{dom, c};
  int n = c.geometry.n, ns = dom ? dom->n_local() : n;
  size_t E = size_t(c.geometry.edge_capacity);
  auto node = [&](const std::string &name, size_t width) { return c.array<float>(name, size_t(n) * width); };
  auto sender_node = [&](const std::string &name, size_t width) { return c.array<float>(name, size_t(ns) * width); };
  const float *cst = m.constants;
  int *status = c.geometry.status;
  int *species = c.array<int>("mh.species", ns);
  energy = node("mh.e", 1), force = sender_node("mh.f", 3), virial = node("mh.v", 9);
  float *x0 = sender_node("mh.embedding", 512);
  DeviceGeometry senders = c.geometry;
  senders.n = ns;
  launch_species(s, senders, m.lookup, species);
  launch_embed(s, ns, species, m.embedding, x0);
  if (ns > n)
    c.clear(force + size_t(3) * n, size_t(ns - n) * 3 * sizeof(float));
  launch_zbl(s, c.geometry, m.constants_dev, m.zbl_radii, m.zbl_c, cst[7], energy, force, virial);
  // Projection path: radial projections on the tensor cores into chunk buffers, tensor
  // products from those (default); otherwise the fused SIMT edge kernels.
  bool projection = projection_edges() && m.layers[0].radial.out && m.layers[1].radial.out;
  if (dom && !projection)
    throw Error("Domain decomposition requires the tensor-core projection path");
  std::vector<ProjectionChunk> chunks;
  long long chunk_cap = 0;
  if (projection) {
    chunks = projection_chunks(c);
    for (auto &k : chunks)
      chunk_cap = std::max(chunk_cap, k.e1 - k.e0);
  }
  EdgeArrays ea{c.array<float>("mh.edge.basis", E * 10), c.array<float>("mh.edge.dbasis", E * 10),
                c.array<float2>("mh.edge.cut", E), c.array<float>("mh.edge.Y", E * 16),
                projection ? c.array<float>("mh.edge.dY", E * 48) : nullptr};
  int *pair = c.array<int>("mh.edge.pair", E);
  launch_edge_geometry(s, c.geometry, species, m.constants_dev, m.radii, m.bessel, ea, pair);
  timer.mark("embedding/ZBL/geometry");
  RadialOut ro[2];
  float *proj[2] = {nullptr, nullptr}; // [R | dR] per layer, chunk_cap rows each
  float *up[2], *rho[2], *raw[2], *res[2], *pin[2], *hidden[2];
  float *msg = node("mh.t.msg", 5120),
        *gate = node("mh.t.gate", 8192), *poly = node("mh.t.poly", 2048), *node_e = node("mh.t.energy", 1);
  const float *input = x0;
  // Both layers' radial MLPs depend on the geometry only: one launch, a grid row per layer
  // (small cells fill twice the SMs of one layer's launch).
  for (int k = 0; k < 2; ++k) {
    std::string p = "mh.l" + std::to_string(k);
    float *hd = c.array<float>(p + ".hd", 2 * E * 64); // h then dh/dr, one GEMM batch apart
    ro[k] = RadialOut{hd, hd + E * 64, c.array<float2>(p + ".den", E)};
  }
  const Layer *radial_layers[2] = {&m.layers[0], &m.layers[1]};
  launch_radial(s, c.geometry, radial_layers, ro, 2, pair, ea, projection);
  timer.mark("radial");
  for (int k = 0; k < 2 && projection; ++k)
    proj[k] = c.array<float>("mh.l" + std::to_string(k) + ".proj",
                             size_t(2 * chunk_cap) * m.layers[k].paths * 128);
  // With one chunk, the projections that depend on the radial rows only -- both layers'
  // (cut h) W and layer 1's r-derivative -- go out as one grouped launch now.  Layer 0's
  // r-derivative waits: its half of the buffer holds the layer-1 up-gradient rows first.
  bool early_projection = projection && chunks.size() == 1;
  if (early_projection) {
    int w0 = m.layers[0].paths * 128, w1 = m.layers[1].paths * 128;
    GemmSpec g[3] = {
        GemmSpec{int(E), w0, 64, 1, ro[0].h, 0, m.layers[0].radial.out, proj[0], w0, 0, false},
        GemmSpec{int(E), w1, 64, 1, ro[1].h, 0, m.layers[1].radial.out, proj[1], w1, 0, false},
        GemmSpec{int(E), w1, 64, 1, ro[1].dh, 0, m.layers[1].radial.out, proj[1] + size_t(chunk_cap) * w1, w1, 0,
                 false}};
    tc_gemm_group(s, g, 3, status);
    timer.mark("projections");
  }
  for (int k = 0; k < 2; ++k) {
    const Layer &l = m.layers[k];
    std::string p = "mh.l" + std::to_string(k);
    up[k] = sender_node(p + ".up", l.in_comp * 128);
    rho[k] = node(p + ".rho", 1);
    raw[k] = node(p + ".raw", 9728);
    res[k] = node(p + ".res", 9728); // kept: the backward recomputes raw / den + res
    pin[k] = node(p + ".pin", 8192);
    hidden[k] = node(p + ".hidden", k ? 512 : 2048);
    int width = l.paths * 128;
    // Layer 0's sender features depend on the element only, so ghosts compute their own;
    // layer 1's come from the ghosts' owners.
    int in_rows = k ? n : ns;
    if (k == 0)
      linear(s, ns, l.up, input, up[k], false, false, status);
    else
      linear(s, n, l.up, input, up[k], false, false, status, n, ns);
    if (dom && k == 1) // overlaps the res / skip linears and the projection
      dom->fetch_ghost_rows(c, up[k], l.in_comp, ns, 128);
    linear(s, n, l.res, up[k], res[k], false, false, status, ns);
    // The skip connection goes straight into the layer output; the product linear adds onto it.
    linear(s, n, l.skip, input, hidden[k], false, false, status, in_rows);
    timer.mark("forward" + std::to_string(k) + ".linears");
    // The messages feed only linear_1: on the projection path and the tensor cores they are
    // written as the GEMM's split operand.
    SplitPlanes ms;
    if (projection && status && linear_takes_split(l.one, false)) {
      ms.hi = reinterpret_cast<uint16_t *>(msg);
      ms.lo = ms.hi + size_t(n) * 5120;
      ms.exp = c.array<int16_t>("mh.t.msg.exp", size_t(n) * 80);
    }
    if (projection) {
      for (auto &q : chunks) {
        // (cut h) W per edge row and path channel; the edge kernel adds cut b.
        if (!early_projection)
          tc_gemm(s, int(q.e1 - q.e0), width, 64, 1, ro[k].h + q.e0 * 64, 0, l.radial.out, proj[k], width, 0,
                  false, status);
        timer.mark("forward" + std::to_string(k) + ".projection");
        if (dom && k == 1 && &q == &chunks.front())
          dom->join(c); // the ghosts' up-projected features have arrived
        launch_message_forward_proj(s, k, c.geometry, l, ea, ro[k], q, proj[k], up[k], msg, rho[k], ns, ms);
        timer.mark("forward" + std::to_string(k) + ".messages");
      }
    } else
      launch_message_forward(s, k, c.geometry, l, ea, ro[k], up[k], msg, rho[k]);
    timer.mark("forward" + std::to_string(k) + ".messages");
    linear(s, n, l.one, msg, raw[k], false, false, status, 0, 0, ms.hi ? &ms : nullptr);
    // The gate feeds only linear_2: on the tensor cores it is written as the GEMM's split
    // operand (the same bytes as fp32, plus one exponent per 64 values), so the GEMM skips
    // its own split.
    SplitPlanes gs;
    if (status && linear_takes_split(l.two, false)) {
      gs.hi = reinterpret_cast<uint16_t *>(gate);
      gs.lo = gs.hi + size_t(n) * 8192;
      gs.exp = c.array<int16_t>("mh.t.gate.exp", size_t(n) * 128);
    }
    launch_normalize_gate(s, n, raw[k], res[k], rho[k], l.alpha, l.beta, cst[11], cst[12], gate, gs);
    timer.mark("forward" + std::to_string(k) + ".node");
    linear(s, n, l.two, gate, pin[k], false, false, status, 0, 0, gs.hi ? &gs : nullptr); // one grouped launch
    timer.mark("forward" + std::to_string(k) + ".linear_2");
    launch_product(s, n, l, pin[k], poly);
    linear(s, n, l.plin, poly, hidden[k], false, true, status);
    if (k == 0) {
      linear(s, n, m.read0, hidden[0], node_e, false, false, status);
      launch_add(s, n, node_e, energy, cst[6]);
    }
    input = hidden[k];
    timer.mark("forward" + std::to_string(k) + ".node");
  }
  float *rpre = node("mh.r.pre", 16), *rhid = node("mh.r.hidden", 16), *rgrad = node("mh.r.grad", 16),
        *rdpre = node("mh.r.dpre", 16);
  linear(s, n, m.read1up, hidden[1], rpre, false, false, status);
  launch_readout_act(s, n * 16, rpre, nullptr, rhid, cst[13], false);
  linear(s, n, m.read1down, rhid, node_e, false, false, status);
  launch_add(s, n, node_e, energy, cst[6]);
  // ---- analytical backward ----
  float *one = node_e;
  float *hgrad1 = node("mh.b.hgrad1", 512), *hgrad0 = node("mh.b.hgrad0", 2048);
  float *pgrad = node("mh.b.poly", 2048), *pingrad = node("mh.b.pin", 8192), *gategrad = gate;
  float *rawgrad = node("mh.b.raw", 9728), *rhograd = node("mh.b.rho", 1);
  float *msggrad = msg, *upgrad = sender_node("mh.b.up", 512);
  float4 *edge_force = c.array<float4>("mh.edge.force", E);
  // Layer-1 up-gradients: every edge's row is written once by the edge backward and summed
  // onto its sender in ascending edge order (no float atomics, reproducible bit for bit).
  // On the projection path the rows reuse the layer-0 dR' half of proj[0], which is free until
  // the layer-0 backward (chunk_cap x 512 floats, exactly one row per chunk edge).
  if (projection && m.layers[0].paths * 128 < 512)
    throw Error("layer-0 projection buffer too small for the up-gradient rows");
  SenderIndex senders_of = build_sender_index(s, c, (long long)E, ns, c.geometry.edge_sender);
  float *ug_edge = projection ? proj[0] + size_t(chunk_cap) * 512 : c.array<float>("mh.edge.ug", E * 512);
  launch_fill(s, n, one, cst[6]);
  linear(s, n, m.read1down, one, rgrad, true, false, status);
  launch_readout_act(s, n * 16, rpre, rgrad, rdpre, cst[13], true);
  linear(s, n, m.read1up, rdpre, hgrad1, true, false, status);
  timer.mark("readouts");
  float *hgrad = hgrad1;
  bool dR0_ready = false; // layer 0's dR' computed early (domain runs overlap it with an exchange)
  for (int k = 1; k >= 0; --k) {
    const Layer &l = m.layers[k];
    if (k == 0)
      linear(s, n, m.read0, one, hgrad, true, true, status);
    linear(s, n, l.plin, hgrad, pgrad, true, false, status);
    // pingrad feeds only the linear_2 backward: on the tensor cores (compiled product tables)
    // layer 1's is written split.  Layer 0's is not: its 410-term table at 64 channels per
    // CTA made the product backward 0.1 ms slower than the GEMM gained (same-box A/B at C3).
    SplitPlanes ps;
    if (k == 1 && status && l.poly_fixed >= 0 && linear_takes_split(l.two, true)) {
      ps.hi = reinterpret_cast<uint16_t *>(pingrad);
      ps.lo = ps.hi + size_t(n) * 8192;
      ps.exp = c.array<int16_t>("mh.b.pin.exp", size_t(n) * 128);
    }
    launch_product_backward(s, n, l, pin[k], pgrad, pingrad, ps);
    linear(s, n, l.two, pingrad, gategrad, true, false, status, 0, 0, ps.hi ? &ps : nullptr);
    float *pregrad = res[k]; // written in place over res[k]
    // rawgrad feeds only the linear_1 backward: on the tensor cores it is written split.
    SplitPlanes rs;
    if (status && linear_takes_split(l.one, true)) {
      rs.hi = reinterpret_cast<uint16_t *>(rawgrad);
      rs.lo = rs.hi + size_t(n) * 9728;
      rs.exp = c.array<int16_t>("mh.b.raw.exp", size_t(n) * 152);
    }
    launch_gate_norm_backward(s, n, res[k], raw[k], rho[k], gategrad, l.alpha, l.beta, cst[11], cst[12], pregrad,
                              rawgrad, rhograd, rs);
    linear(s, n, l.one, rawgrad, msggrad, true, false, status, 0, 0, rs.hi ? &rs : nullptr);
    if (k == 1) {
      if (dom) { // ghost rows collect the edge kernels' up-gradients for their owners
        c.clear(upgrad, size_t(ns) * 512 * sizeof(float));
        linear(s, n, l.res, pregrad, upgrad, true, true, status, n, ns);
      } else {
        linear(s, n, l.res, pregrad, upgrad, true, false, status);
      }
    }
    timer.mark("backward" + std::to_string(k) + ".node");
    if (projection) {
      int width = l.paths * 128;
      float *R = proj[k], *dR = proj[k] + size_t(chunk_cap) * width;
      for (auto &q : chunks) {
        int rows = int(q.e1 - q.e0);
        // (cut dh + dcut h) W; with several chunks, (cut h) W is recomputed beside it.
        if (chunks.size() == 1) { // (cut h) W is still in place from the forward pass
          if (!(k == 0 && dR0_ready) && !(k == 1 && early_projection))
            tc_gemm(s, rows, width, 64, 1, ro[k].dh + q.e0 * 64, 0, l.radial.out, dR, width, 0, false, status);
        }
        else
          tc_gemm(s, rows, width, 64, 2, ro[k].h + q.e0 * 64, (long long)E * 64, l.radial.out, R, width,
                  (long long)chunk_cap * width, false, status);
        timer.mark("backward" + std::to_string(k) + ".projection");
        launch_message_backward_proj(s, k, c.geometry, l, ea, ro[k], q, R, dR, up[k], msggrad, rhograd, ug_edge,
                                     edge_force, k == 0, ns);
        timer.mark("backward" + std::to_string(k) + ".edges");
        if (k == 1) {
          launch_sender_gather(s, senders_of, q.e0, q.e1, ug_edge, 4, upgrad, ns);
          timer.mark("backward1.sender-gather");
        }
      }
    } else {
      launch_message_backward(s, k, c.geometry, l, ea, ro[k], up[k], msggrad, rhograd, ug_edge, edge_force, k == 0);
      if (k == 1)
        launch_sender_gather(s, senders_of, 0, (long long)E, ug_edge, 4, upgrad, ns);
    }
    timer.mark("backward" + std::to_string(k) + ".edges");
    if (k == 1) {
      if (dom)
        dom->return_ghost_rows(c, upgrad, l.in_comp, ns, 128);
      // Independent of the returned gradients: overlaps their exchange.
      linear(s, n, l.skip, hgrad, hgrad0, true, false, status);
      if (dom && projection && chunks.size() == 1) {
        // Layer 0's (cut dh + dcut h) W now: the up-gradient rows it overwrites are consumed.
        const Layer &l0 = m.layers[0];
        int width0 = l0.paths * 128;
        tc_gemm(s, int(chunks[0].e1 - chunks[0].e0), width0, 64, 1, ro[0].dh, 0, l0.radial.out,
                proj[0] + size_t(chunk_cap) * width0, width0, 0, false, status);
        dR0_ready = true;
      }
      if (dom)
        dom->join(c);
      linear(s, n, l.up, upgrad, hgrad0, true, true, status, ns, n);
      hgrad = hgrad0;
    }
  }
  if (dom) {
    launch_force_gather_domain(s, c.geometry, edge_force, force, virial);
    launch_ghost_reactions(s, senders_of, n, edge_force, force);
    dom->return_ghost_rows(c, force, 1, ns, 3);
    dom->join(c);
  } else {
    launch_force_gather(s, c.geometry, edge_force, force, virial);
  }
  check(cudaGetLastError());
  timer.mark("forces");
  if (dom) {
    // Every rank's owned rows into full-structure arrays, summed over ranks.
    float *out = c.array<float>("mh.domain.out", size_t(n_full) * 13);
    dom->gather_outputs(c, energy, force, virial, out, out + n_full, out + size_t(4) * n_full);
    dom->restore(c);
    restore_geometry.d = nullptr;
    energy = out;
    force = out + n_full;
    virial = out + size_t(4) * n_full;
  }
  };
  if (record) {
    // Capture (nothing runs), then launch the graph.  Any failure -- a call that cannot be
    // captured -- ends the capture and falls back to launching the kernels directly.
    gc.drop();
    cudaGraph_t graph = nullptr;
    bool ok = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
    if (ok) {
      try {
        enqueue();
      } catch (...) {
        ok = false;
      }
      ok = cudaStreamEndCapture(s, &graph) == cudaSuccess && ok && graph;
      if (ok)
        ok = cudaGraphInstantiateWithFlags(&gc.exec, graph, 0) == cudaSuccess;
      if (graph)
        cudaGraphDestroy(graph);
    }
    if (ok) {
      gc.recorded.set(c);
      gc.energy = energy, gc.force = force, gc.virial = virial;
      gc.launches = launch_counter() - launches_before;
      c.diagnostics.graph = "recorded";
      check(cudaGraphLaunch(gc.exec, s));
    } else {
      cudaGetLastError(); // clear a capture error; run the same work directly
      gc.drop();
      gc.seen.valid = false;
      launch_counter() = launches_before;
      enqueue();
    }
  } else {
    enqueue();
  }
  auto results = finish();
  c.diagnostics.launches = launch_counter();
  return results;
}
} // namespace mace
