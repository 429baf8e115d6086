// Spatial domain decomposition across ranks over NCCL (see include/lapis/domain.hpp).
//
// Ownership: rank r owns the internal (bin-sorted) atoms [n r / W, n (r + 1) / W) -- a compact
// slab, since bins are ordered with their first lattice index slowest.  Context::prepare is
// partitioned the same way (Context::part / parts): it wraps and bins every atom (O(n), so
// the internal order is the same on every rank) but builds CSR rows only for this rank's
// receivers, so the edge arrays of a rank hold its own edges only.
//
// The exchange plan is derived from the local rows alone.  Ghosts are the foreign senders of
// this rank's edges, numbered after the owned atoms in ascending internal id (so the ghosts of
// one owner form one block).  The atoms this rank sends to peer r are its receivers that have
// an edge from one of r's atoms: the edge relation is symmetric (every edge j <- i has its
// reverse i <- j; prepare checks this for edges between owned atoms), so that set equals r's
// ghost block for this rank, in the same ascending order, and no request messages are needed.
// Before the first exchange of every call, the ranks all-gather their plan sizes and the
// structure they were given; a mismatch fails the call on every rank (before any exchange
// that could wait forever).
//
// Failure handling: the communicator is created non-blocking (ncclCommInitRankConfig with
// blocking = 0).  Every host-side NCCL step and every wait for the device (the exchanges run
// on the model stream) polls with a deadline (MACE_DOMAIN_TIMEOUT_S, default 120 s).  On
// expiry, or on an asynchronous NCCL error, the communicator is aborted (ncclCommAbort, which
// also ends NCCL kernels still waiting on a peer), the domain is marked failed and the call
// throws; later calls on it throw at once.
#include "lapis/domain.hpp"
#include "launch.cuh"
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <dlfcn.h>
#include <mutex>
#include <thread>
#include <vector>

namespace lapis {
namespace {
// ---------------- NCCL, loaded at run time ----------------
struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
};

const Nccl &nccl() {
  static Nccl n;
  static std::once_flag once;
  static std::string failure;
  std::call_once(once, [] {
    // Prefer a libnccl already loaded in the process (e.g. by torch), else load the system one.
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h)
      h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      failure = "NCCL (libnccl.so.2) could not be loaded";
      return;
    }
    auto sym = [&](auto &fn, const char *name) { fn = reinterpret_cast<std::decay_t<decltype(fn)>>(dlsym(h, name)); };
    sym(n.get_unique_id, "ncclGetUniqueId");
    sym(n.comm_init_rank_config, "ncclCommInitRankConfig");
    sym(n.comm_destroy, "ncclCommDestroy");
    sym(n.comm_abort, "ncclCommAbort");
    sym(n.comm_get_async_error, "ncclCommGetAsyncError");
    sym(n.send, "ncclSend");
    sym(n.recv, "ncclRecv");
    sym(n.all_reduce, "ncclAllReduce");
    sym(n.all_gather, "ncclAllGather");
    sym(n.group_start, "ncclGroupStart");
    sym(n.group_end, "ncclGroupEnd");
    sym(n.error_string, "ncclGetErrorString");
    if (!n.get_unique_id || !n.comm_init_rank_config || !n.comm_destroy || !n.comm_abort ||
        !n.comm_get_async_error || !n.send || !n.recv || !n.all_reduce || !n.all_gather || !n.group_start ||
        !n.group_end || !n.error_string)
      failure = "libnccl.so.2 lacks a required symbol";
  });
  if (!failure.empty())
    throw Error(failure);
  return n;
}

double timeout_seconds() {
  static const double s = [] {
    const char *v = std::getenv("MACE_DOMAIN_TIMEOUT_S");
    double t = v ? std::atof(v) : 0;
    return t > 0 ? t : 120.0;
  }();
  return s;
}

// ---------------- plan kernels ----------------
// flag[j] = 1 for every foreign sender j (outside [o0, o1)) of the local edges.
__global__ void mark_foreign_senders(long long E, const int *sender, int o0, int o1, int *flag) {
  long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (e < E) {
    int j = sender[e];
    if (j < o0 || j >= o1)
      flag[j] = 1;
  }
}
// Thread per local receiver w: peer[r * n_own + w] = 1 if w has an edge from an atom of rank r
// (r != this rank).  starts: the W + 1 ownership bounds.
__global__ void mark_peer_receivers(int n_own, int world, int me, const int *row, const int *sender,
                                    const int *starts, int *peer) {
  int w = blockIdx.x * blockDim.x + threadIdx.x;
  if (w >= n_own)
    return;
  for (int e = row[w]; e < row[w + 1]; ++e) {
    int j = sender[e], r = 0;
    while (r + 1 < world && j >= starts[r + 1])
      ++r;
    if (r != me)
      peer[size_t(r) * n_own + w] = 1;
  }
}
// Exclusive scan of n flags by one CTA; out[n] = total.
__global__ void scan_flags(const int *in, int *out, int n) {
  __shared__ int partial[1024];
  int t = threadIdx.x;
  int chunk = (n + 1023) / 1024, begin = min(n, t * chunk), end = min(n, begin + chunk), s = 0;
  for (int k = begin; k < end; ++k)
    s += in[k];
  partial[t] = s;
  __syncthreads();
  for (int step = 1; step < 1024; step *= 2) {
    int v = t >= step ? partial[t - step] : 0;
    __syncthreads();
    partial[t] += v;
    __syncthreads();
  }
  int run = t ? partial[t - 1] : 0;
  for (int k = begin; k < end; ++k) {
    out[k] = run;
    run += in[k];
  }
  if (t == 1023)
    out[n] = partial[1023];
}
// out[r] = ghost_pos[starts[r]] (r <= W), out[W + 1 + r] = peer r's send total.
__global__ void plan_sizes(int world, int n_own, const int *ghost_pos, const int *starts, const int *ppos, int *out) {
  for (int r = threadIdx.x; r <= world; r += blockDim.x)
    out[r] = ghost_pos[starts[r]];
  for (int r = threadIdx.x; r < world; r += blockDim.x)
    out[world + 1 + r] = ppos[size_t(r) * (n_own + 1) + n_own];
}
__global__ void compact(int n, const int *flag, const int *pos, int base, int *list) {
  int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j < n && flag[j])
    list[pos[j]] = j + base;
}
// Local sender numbering: owned atoms [0, n_own), ghosts n_own + their rank in the ghost list.
__global__ void local_senders(long long E, const int *sender, int o0, int o1, int n_own, const int *ghost_pos,
                              int *lsender) {
  long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (e < E) {
    int j = sender[e];
    lsender[e] = j >= o0 && j < o1 ? j - o0 : n_own + ghost_pos[j];
  }
}
__global__ void local_elements(int n_own, int n_ghost, int o0, const int *elements, const int *ghosts, int *out) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n_own)
    out[i] = elements[o0 + i];
  else if (i < n_own + n_ghost)
    out[i] = elements[ghosts[i - n_own]];
}
// buf[k][c][w] = x[(c * stride + rows[k]) * width + w]
__global__ void pack_rows(int count, int comps, int stride, int width, const int *rows, int row_base, const float *x,
                          float *buf) {
  long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  long long total = (long long)count * comps * width;
  if (q >= total)
    return;
  int w = int(q % width), c = int((q / width) % comps), k = int(q / ((long long)width * comps));
  int row = rows ? rows[k] : row_base + k;
  buf[q] = x[(size_t(c) * stride + row) * width + w];
}
// x[(c * stride + rows[k]) * width + w] (+)= buf[k][c][w]
__global__ void unpack_rows(int count, int comps, int stride, int width, const int *rows, int row_base,
                            const float *buf, float *x, int add) {
  long long q = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  long long total = (long long)count * comps * width;
  if (q >= total)
    return;
  int w = int(q % width), c = int((q / width) % comps), k = int(q / ((long long)width * comps));
  int row = rows ? rows[k] : row_base + k;
  float *dst = x + (size_t(c) * stride + row) * width + w;
  *dst = add ? *dst + buf[q] : buf[q];
}
__global__ void place_owned(int n_own, int o0, const float *e, const float *f, const float *v, float *ef, float *ff,
                            float *vf) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_own)
    return;
  ef[o0 + i] = e[i];
  for (int k = 0; k < 3; ++k)
    ff[3 * (o0 + i) + k] = f[3 * i + k];
  for (int k = 0; k < 9; ++k)
    vf[9 * (o0 + i) + k] = v[9 * i + k];
}

inline int blocks(long long n, int t = 256) { return int(std::max<long long>(1, (n + t - 1) / t)); }

// FNV-1a over the bytes of the cell (float32) and the atom count: ranks given different
// structures are told apart before they exchange anything.
unsigned structure_tag(int n, const float *h) {
  unsigned x = 2166136261u;
  auto mix = [&](const void *p, size_t bytes) {
    for (size_t k = 0; k < bytes; ++k)
      x = (x ^ static_cast<const unsigned char *>(p)[k]) * 16777619u;
  };
  mix(&n, sizeof n);
  mix(h, 9 * sizeof(float));
  return x;
}
} // namespace

std::string nccl_unique_id() {
  ncclUniqueId id;
  ncclResult_t r = nccl().get_unique_id(&id);
  if (r != ncclSuccess)
    throw Error(std::string("ncclGetUniqueId: ") + nccl().error_string(r));
  return std::string(id.internal, sizeof(id.internal));
}

struct ExchangePlan {
  std::vector<int> starts;                             // [world + 1] ownership bounds
  int o0 = 0, o1 = 0, n_own = 0, n_local = 0;
  std::vector<int> send_count, ghost_off, ghost_count; // per peer
  std::vector<int *> send_list;                        // per peer: local row ids (device)
  int *ghosts = nullptr;                               // [n_local - n_own] internal ids (device)
  int *ghost_pos = nullptr;                            // [n + 1] ghost rank of each atom (device)
};

struct Domain::Impl {
  int rank, world;
  ncclComm_t comm = nullptr;
  bool failed = false;
  std::string failure;
  DeviceGeometry full{};
  bool localized = false;
  int n_own = 0, n_local = 0, o0 = 0, o1 = 0;
  long long calls = 0;
  std::vector<int> starts;                             // [world + 1] ownership ranges (internal ids)
  std::vector<int> send_count, ghost_off, ghost_count; // per peer
  std::vector<int *> send_list;                        // per peer: local row ids to send (device)
  cudaEvent_t done = nullptr;
  // Every NCCL operation runs on `exchange`, a stream of the domain: the model stream hands
  // over with `ready` and waits for `finished` only where it needs the result (join), so the
  // transfers overlap the model's independent work.
  cudaStream_t exchange = nullptr;
  cudaEvent_t ready = nullptr, finished = nullptr;
  void hand_over(cudaStream_t from) {
    check(cudaEventRecord(ready, from));
    check(cudaStreamWaitEvent(exchange, ready, 0));
  }
  void mark_finished() { check(cudaEventRecord(finished, exchange)); }

  // The communicator becomes unusable: abort it (which also releases NCCL kernels that wait
  // on a peer) and remember why.
  [[noreturn]] void fail(const std::string &why) {
    if (comm && !failed)
      nccl().comm_abort(comm);
    comm = nullptr;
    failed = true;
    failure = why;
    throw Error(why);
  }
  void check_usable() const {
    if (failed)
      throw Error("Domain communicator failed earlier: " + failure);
  }
  // Polling back-off: yield for the first ~20,000 polls (tens of microseconds to a few
  // milliseconds -- the usual wait, where a sleep would leave the GPU idle), then sleep 50 us.
  static void pause(long long spins) {
    if (spins < 20000)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  // Host side of a non-blocking NCCL step: the call itself, then its completion state polled
  // until it leaves ncclInProgress (deadline: the domain timeout).
  void step(ncclResult_t r, const char *what) {
    const auto &N = nccl();
    if (r != ncclSuccess && r != ncclInProgress)
      fail(std::string(what) + ": " + N.error_string(r));
    auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_seconds());
    long long spins = 0;
    for (;;) {
      ncclResult_t st = ncclSuccess;
      ncclResult_t q = N.comm_get_async_error(comm, &st);
      if (q != ncclSuccess)
        fail(std::string(what) + ": ncclCommGetAsyncError: " + N.error_string(q));
      if (st == ncclSuccess)
        return;
      if (st != ncclInProgress)
        fail(std::string(what) + ": " + N.error_string(st));
      if (std::chrono::steady_clock::now() > deadline)
        fail(std::string(what) + ": timed out after " + std::to_string(timeout_seconds()) + " s");
      pause(spins++);
    }
  }
  // Waits for the work enqueued so far on `s` (the exchanges included) with the domain
  // deadline, watching for asynchronous NCCL errors meanwhile.
  void wait(cudaStream_t s, const char *what) {
    const auto &N = nccl();
    check(cudaEventRecord(done, s));
    auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_seconds());
    long long spins = 0;
    for (;;) {
      cudaError_t q = cudaEventQuery(done);
      if (q == cudaSuccess)
        return;
      if (q != cudaErrorNotReady)
        check(q);
      ncclResult_t st = ncclSuccess;
      if (N.comm_get_async_error(comm, &st) != ncclSuccess || (st != ncclSuccess && st != ncclInProgress))
        fail(std::string(what) + ": NCCL reported " + N.error_string(st));
      if (std::chrono::steady_clock::now() > deadline)
        fail(std::string(what) + ": a peer did not take part within " + std::to_string(timeout_seconds()) +
             " s (MACE_DOMAIN_TIMEOUT_S)");
      pause(spins++);
    }
  }
};

Domain::Domain(int rank, int world, const void *unique_id) : impl_(std::make_unique<Impl>()) {
  if (world < 1 || world > 1024 || rank < 0 || rank >= world || !unique_id)
    throw Error("Invalid domain rank or size");
  auto &d = *impl_;
  d.rank = rank;
  d.world = world;
  check(cudaEventCreateWithFlags(&d.done, cudaEventDisableTiming));
  check(cudaEventCreateWithFlags(&d.ready, cudaEventDisableTiming));
  check(cudaEventCreateWithFlags(&d.finished, cudaEventDisableTiming));
  check(cudaStreamCreateWithFlags(&d.exchange, cudaStreamNonBlocking));
  ncclUniqueId id;
  std::copy(static_cast<const char *>(unique_id), static_cast<const char *>(unique_id) + sizeof(id.internal),
            id.internal);
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  ncclResult_t r = nccl().comm_init_rank_config(&d.comm, world, id, rank, &config);
  d.step(r, "ncclCommInitRankConfig");
}
Domain::~Domain() {
  if (!impl_)
    return;
  if (impl_->comm) {
    // A clean communicator is destroyed; if its last step did not finish, abort instead.
    ncclResult_t st = ncclSuccess;
    if (nccl().comm_get_async_error(impl_->comm, &st) == ncclSuccess && st == ncclSuccess)
      nccl().comm_destroy(impl_->comm);
    else
      nccl().comm_abort(impl_->comm);
  }
  if (impl_->done)
    cudaEventDestroy(impl_->done);
  if (impl_->ready)
    cudaEventDestroy(impl_->ready);
  if (impl_->finished)
    cudaEventDestroy(impl_->finished);
  if (impl_->exchange)
    cudaStreamDestroy(impl_->exchange);
}
int Domain::rank() const { return impl_->rank; }
int Domain::world() const { return impl_->world; }
int Domain::n_own() const { return impl_->n_own; }
int Domain::n_local() const { return impl_->n_local; }
void Domain::partition(Context &ctx) const {
  impl_->check_usable();
  ctx.part = impl_->rank;
  ctx.parts = impl_->world;
}

// The exchange plan of `rank` among `world` from the context's partitioned rows (device lists,
// host sizes).  Shared by Domain::localize and the single-GPU plan check
// (lapis_exchange_plan_device).
ExchangePlan build_plan(Context &ctx, int rank, int world) {
  const DeviceGeometry &g = ctx.geometry;
  int n = g.n, W = world;
  cudaStream_t s = ctx.stream;
  ExchangePlan p;
  p.starts.assign(W + 1, 0);
  for (int r = 0; r <= W; ++r)
    p.starts[r] = int((long long)n * r / W);
  p.o0 = p.starts[rank];
  p.o1 = p.starts[rank + 1];
  p.n_own = p.o1 - p.o0;
  if (g.receiver_begin != p.o0 || g.receiver_count != p.n_own)
    throw Error("Domain: the context was not prepared for this rank's receivers");
  long long E = g.edge_capacity;
  // Ghosts: foreign senders of this rank's edges, ascending internal id.
  int *flag = ctx.array<int>("domain.flag", size_t(n) + 1);
  p.ghost_pos = ctx.array<int>("domain.pos", size_t(n) + 1);
  ctx.clear(flag, size_t(n + 1) * sizeof(int));
  if (E)
    lapis::launch(mark_foreign_senders, blocks(E), 256, 0, s, E, g.edge_sender, p.o0, p.o1, flag);
  lapis::launch(scan_flags, 1, 1024, 0, s, flag, p.ghost_pos, n);
  // Sends: this rank's receivers with an edge from each peer.
  int *starts = ctx.array<int>("domain.starts", size_t(W) + 1);
  int *peer = ctx.array<int>("domain.peer", size_t(W) * std::max(p.n_own, 1));
  int *ppos = ctx.array<int>("domain.peer_pos", size_t(W) * (size_t(p.n_own) + 1));
  check(cudaMemcpyAsync(starts, p.starts.data(), size_t(W + 1) * sizeof(int), cudaMemcpyHostToDevice, s));
  ctx.clear(peer, size_t(W) * std::max(p.n_own, 1) * sizeof(int));
  if (p.n_own)
    lapis::launch(mark_peer_receivers, blocks(p.n_own), 256, 0, s, p.n_own, W, rank, g.edge_offsets, g.edge_sender,
                  starts, peer);
  for (int r = 0; r < W; ++r)
    lapis::launch(scan_flags, 1, 1024, 0, s, peer + size_t(r) * p.n_own, ppos + size_t(r) * (p.n_own + 1), p.n_own);
  // Plan sizes (host, one copy): ghost block offsets at the ownership bounds, send totals per
  // peer.
  int *sizes = ctx.array<int>("domain.sizes", 2 * size_t(W) + 1);
  lapis::launch(plan_sizes, 1, 64, 0, s, W, p.n_own, p.ghost_pos, starts, ppos, sizes);
  std::vector<int> host_sizes(2 * W + 1);
  check(cudaMemcpyAsync(host_sizes.data(), sizes, host_sizes.size() * sizeof(int), cudaMemcpyDeviceToHost, s));
  check(cudaStreamSynchronize(s)); // local work only: no peer is involved
  const int *pos_at = host_sizes.data(), *sends = host_sizes.data() + W + 1;
  int n_ghost = pos_at[W];
  p.n_local = p.n_own + n_ghost;
  p.ghost_off.assign(W, 0);
  p.ghost_count.assign(W, 0);
  p.send_count.assign(W, 0);
  for (int r = 0; r < W; ++r) {
    p.ghost_off[r] = pos_at[r];
    p.ghost_count[r] = r == rank ? 0 : pos_at[r + 1] - pos_at[r];
    p.send_count[r] = r == rank ? 0 : sends[r];
  }
  p.ghosts = ctx.array<int>("domain.ghosts", std::max(n_ghost, 1));
  lapis::launch(compact, blocks(n), 256, 0, s, n, flag, p.ghost_pos, 0, p.ghosts);
  p.send_list.assign(W, nullptr);
  for (int r = 0; r < W; ++r) {
    if (r == rank)
      continue;
    p.send_list[r] = ctx.array<int>("domain.send." + std::to_string(r), std::max(p.send_count[r], 1));
    if (p.n_own)
      lapis::launch(compact, blocks(p.n_own), 256, 0, s, p.n_own, peer + size_t(r) * p.n_own,
                    ppos + size_t(r) * (p.n_own + 1), 0, p.send_list[r]);
  }
  check(cudaGetLastError());
  return p;
}

void Domain::localize(Context &ctx) {
  auto &d = *impl_;
  d.check_usable();
  const DeviceGeometry &g = ctx.geometry;
  int n = g.n, W = d.world;
  cudaStream_t s = ctx.stream;
  ExchangePlan p = build_plan(ctx, d.rank, W);
  d.starts = p.starts;
  d.o0 = p.o0;
  d.o1 = p.o1;
  d.n_own = p.n_own;
  d.n_local = p.n_local;
  d.ghost_off = p.ghost_off;
  d.ghost_count = p.ghost_count;
  d.send_count = p.send_count;
  d.send_list = p.send_list;
  d.full = g;
  // Consistency check across ranks: structure tag, call count, and the plan sizes.  Peer r's
  // sends to this rank must equal this rank's ghost block from r, for every pair.
  const int fields = 3 + 2 * W;
  std::vector<int> mine(fields), all(size_t(fields) * W);
  mine[0] = n;
  mine[1] = int(structure_tag(n, g.h));
  mine[2] = int(d.calls);
  for (int r = 0; r < W; ++r) {
    mine[3 + r] = d.send_count[r];
    mine[3 + W + r] = d.ghost_count[r];
  }
  int *dmine = ctx.array<int>("domain.check", size_t(fields) * (W + 1));
  check(cudaMemcpyAsync(dmine, mine.data(), size_t(fields) * sizeof(int), cudaMemcpyHostToDevice, s));
  if (W > 1) {
    d.hand_over(s);
    d.step(nccl().all_gather(dmine, dmine + fields, size_t(fields), ncclInt32, d.comm, d.exchange), "ncclAllGather");
    d.wait(d.exchange, "domain plan check");
    check(cudaMemcpy(all.data(), dmine + fields, all.size() * sizeof(int), cudaMemcpyDeviceToHost));
  } else {
    all = mine;
  }
  ++d.calls;
  for (int r = 0; r < W; ++r) {
    const int *o = all.data() + size_t(r) * fields;
    if (o[0] != n || o[1] != mine[1] || o[2] != mine[2])
      throw Error("Domain: ranks were given different structures or calls (rank " + std::to_string(r) + ")");
    for (int q = 0; q < W; ++q) {
      const int *pq = all.data() + size_t(q) * fields;
      if (o[3 + q] != pq[3 + W + r])
        throw Error("Domain: exchange plan mismatch between ranks " + std::to_string(r) + " and " +
                    std::to_string(q) + " (asymmetric edge set?)");
    }
  }
  // The local graph: owned receivers (the prepared rows), senders renumbered.
  long long E = g.edge_capacity;
  int n_ghost = p.n_local - p.n_own;
  int *lsender = ctx.array<int>("domain.sender", size_t(std::max<long long>(E, 1)));
  int *lz = ctx.array<int>("domain.elements", std::max(d.n_local, 1));
  if (E)
    lapis::launch(local_senders, blocks(E), 256, 0, s, E, g.edge_sender, d.o0, d.o1, d.n_own, p.ghost_pos, lsender);
  lapis::launch(local_elements, blocks(d.n_local), 256, 0, s, d.n_own, n_ghost, d.o0, g.elements, p.ghosts, lz);
  check(cudaGetLastError());
  DeviceGeometry l = g;
  l.n = d.n_own;
  l.elements = lz;
  l.edge_sender = lsender;
  l.receiver_begin = 0;
  l.receiver_count = d.n_own;
  ctx.geometry = l;
  d.localized = true;
}

void Domain::restore(Context &ctx) {
  if (impl_->localized)
    ctx.geometry = impl_->full;
  impl_->localized = false;
}

void Domain::fetch_ghost_rows(Context &ctx, float *x, int comps, int stride, int width) {
  auto &d = *impl_;
  d.check_usable();
  const auto &N = nccl();
  cudaStream_t s = d.exchange;
  d.hand_over(ctx.stream);
  std::vector<float *> sbuf(d.world, nullptr), rbuf(d.world, nullptr);
  for (int r = 0; r < d.world; ++r) {
    if (r == d.rank)
      continue;
    size_t sn = size_t(d.send_count[r]) * comps * width, rn = size_t(d.ghost_count[r]) * comps * width;
    sbuf[r] = ctx.array<float>("domain.sbuf." + std::to_string(r), std::max<size_t>(sn, 1));
    rbuf[r] = ctx.array<float>("domain.rbuf." + std::to_string(r), std::max<size_t>(rn, 1));
    if (sn)
      lapis::launch(pack_rows, blocks((long long)sn), 256, 0, s, d.send_count[r], comps, stride, width, d.send_list[r],
                    0, x, sbuf[r]);
  }
  d.step(N.group_start(), "ncclGroupStart");
  for (int r = 0; r < d.world; ++r) {
    if (r == d.rank)
      continue;
    if (d.send_count[r])
      d.step(N.send(sbuf[r], size_t(d.send_count[r]) * comps * width, ncclFloat32, r, d.comm, s), "ncclSend");
    if (d.ghost_count[r])
      d.step(N.recv(rbuf[r], size_t(d.ghost_count[r]) * comps * width, ncclFloat32, r, d.comm, s), "ncclRecv");
  }
  d.step(N.group_end(), "ncclGroupEnd");
  for (int r = 0; r < d.world; ++r)
    if (r != d.rank && d.ghost_count[r])
      lapis::launch(unpack_rows, blocks((long long)d.ghost_count[r] * comps * width), 256, 0, s, d.ghost_count[r], comps,
                    stride, width, static_cast<const int *>(nullptr), d.n_own + d.ghost_off[r], rbuf[r], x, 0);
  d.mark_finished();
}

void Domain::return_ghost_rows(Context &ctx, float *x, int comps, int stride, int width) {
  auto &d = *impl_;
  d.check_usable();
  const auto &N = nccl();
  cudaStream_t s = d.exchange;
  d.hand_over(ctx.stream);
  std::vector<float *> sbuf(d.world, nullptr), rbuf(d.world, nullptr);
  for (int r = 0; r < d.world; ++r) {
    if (r == d.rank)
      continue;
    size_t sn = size_t(d.ghost_count[r]) * comps * width, rn = size_t(d.send_count[r]) * comps * width;
    sbuf[r] = ctx.array<float>("domain.sbuf." + std::to_string(r), std::max<size_t>(sn, 1));
    rbuf[r] = ctx.array<float>("domain.rbuf." + std::to_string(r), std::max<size_t>(rn, 1));
    if (sn)
      lapis::launch(pack_rows, blocks((long long)sn), 256, 0, s, d.ghost_count[r], comps, stride, width,
                    static_cast<const int *>(nullptr), d.n_own + d.ghost_off[r], x, sbuf[r]);
  }
  d.step(N.group_start(), "ncclGroupStart");
  for (int r = 0; r < d.world; ++r) {
    if (r == d.rank)
      continue;
    if (d.ghost_count[r])
      d.step(N.send(sbuf[r], size_t(d.ghost_count[r]) * comps * width, ncclFloat32, r, d.comm, s), "ncclSend");
    if (d.send_count[r])
      d.step(N.recv(rbuf[r], size_t(d.send_count[r]) * comps * width, ncclFloat32, r, d.comm, s), "ncclRecv");
  }
  d.step(N.group_end(), "ncclGroupEnd");
  // Added in rank order: a fixed order per atom.
  for (int r = 0; r < d.world; ++r)
    if (r != d.rank && d.send_count[r])
      lapis::launch(unpack_rows, blocks((long long)d.send_count[r] * comps * width), 256, 0, s, d.send_count[r], comps,
                    stride, width, static_cast<const int *>(d.send_list[r]), 0, rbuf[r], x, 1);
  d.mark_finished();
}

void Domain::join(Context &ctx) {
  auto &d = *impl_;
  check(cudaStreamWaitEvent(ctx.stream, d.finished, 0));
}

void Domain::gather_outputs(Context &ctx, const float *e, const float *f, const float *v, float *ef, float *ff,
                            float *vf) {
  auto &d = *impl_;
  d.check_usable();
  cudaStream_t s = ctx.stream;
  int n = d.full.n;
  // ef, ff, vf are one contiguous [13 n] buffer: zero, place the owned rows, sum over ranks.
  ctx.clear(ef, size_t(n) * 13 * sizeof(float));
  if (d.n_own)
    lapis::launch(place_owned, blocks(d.n_own), 256, 0, s, d.n_own, d.o0, e, f, v, ef, ff, vf);
  if (d.world > 1) {
    d.hand_over(s);
    d.step(nccl().all_reduce(ef, ef, size_t(n) * 13, ncclFloat32, ncclSum, d.comm, d.exchange), "ncclAllReduce");
    d.mark_finished();
    check(cudaStreamWaitEvent(s, d.finished, 0));
    d.wait(s, "domain output all-reduce");
  }
}
} // namespace lapis

// ---------------------------------------------------------------------------------------
// Single-GPU view of one rank's exchange plan (no communicator): the partitioned neighbour
// list and the plan kernels of a decomposed evaluation, for checks against the host rules
// (lapis_exchange_plan_host) and across ranks.
// ---------------------------------------------------------------------------------------
#include "mace/c_api.h"

namespace lapis {
void set_c_api_error(const std::string &message);
}

long long lapis_exchange_plan(int n, const float *xyz, const float *cell, float cutoff, int rank, int world,
                              int *send_counts, int *ghost_counts, int *internal_to_input, int *row, int *sender,
                              int *ghosts, int *sends, long long capacity) {
  using namespace lapis;
  try {
    set_c_api_error("");
    if (n < 0 || !cell || (n && !xyz) || world < 1 || rank < 0 || rank >= world || !send_counts || !ghost_counts)
      throw Error("Invalid exchange-plan arguments");
    std::vector<int> z(size_t(n), 1);
    Structure s;
    s.size = n;
    s.positions = xyz;
    s.elements = z.data();
    std::copy(cell, cell + 9, s.cell.begin());
    Context ctx;
    ctx.part = rank;
    ctx.parts = world;
    ctx.prepare(s, cutoff, Options{});
    ctx.synchronize();
    ExchangePlan p = build_plan(ctx, rank, world);
    const DeviceGeometry &g = ctx.geometry;
    long long E = g.edge_capacity;
    std::copy(p.send_count.begin(), p.send_count.end(), send_counts);
    std::copy(p.ghost_count.begin(), p.ghost_count.end(), ghost_counts);
    if (capacity >= std::max<long long>(E, n)) {
      if (!internal_to_input || !row || !sender || !ghosts || !sends)
        throw Error("Null exchange-plan outputs");
      check(cudaMemcpy(internal_to_input, ctx.internal_to_original, size_t(n) * sizeof(int), cudaMemcpyDeviceToHost));
      check(cudaMemcpy(row, g.edge_offsets, (size_t(p.n_own) + 1) * sizeof(int), cudaMemcpyDeviceToHost));
      check(cudaMemcpy(sender, g.edge_sender, size_t(E) * sizeof(int), cudaMemcpyDeviceToHost));
      check(cudaMemcpy(ghosts, p.ghosts, size_t(p.n_local - p.n_own) * sizeof(int), cudaMemcpyDeviceToHost));
      size_t k = 0;
      for (int q = 0; q < world; ++q) {
        if (q == rank || !p.send_count[q])
          continue;
        check(cudaMemcpy(sends + k, p.send_list[q], size_t(p.send_count[q]) * sizeof(int), cudaMemcpyDeviceToHost));
        for (int t = 0; t < p.send_count[q]; ++t)
          sends[k + t] += p.o0; // local rows -> internal ids
        k += size_t(p.send_count[q]);
      }
    }
    return E;
  } catch (const std::exception &e) {
    set_c_api_error(e.what());
    return -1;
  }
}
