// Spatial domain decomposition across ranks over NCCL (see include/lapis/domain.hpp).
//
// Ownership: rank r owns the internal (bin-sorted) atoms [n r / W, n (r + 1) / W) -- a compact
// slab, since bins are ordered with their first lattice index slowest -- and therefore the
// contiguous CSR edge range of those receivers.  Ghosts are the senders of those edges that
// another rank owns, numbered after the owned atoms in ascending internal id, so the ghosts of
// one owner form one contiguous block.  Every rank derives what each peer needs from it
// (the owned senders of that peer's edges) from the full edge list it already holds, so no
// request messages are exchanged: the send list for peer s and s's ghost block for this rank
// are the same atoms in the same (ascending) order.
#include "lapis/domain.hpp"
#include "launch.cuh"
#include <nccl.h>

#include <algorithm>
#include <dlfcn.h>
#include <mutex>
#include <vector>

namespace lapis {
namespace {
// ---------------- NCCL, loaded at run time ----------------
struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
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
    auto sym = [&](const char *name) { return dlsym(h, name); };
    n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(sym("ncclGetUniqueId"));
    n.comm_init_rank = reinterpret_cast<decltype(n.comm_init_rank)>(sym("ncclCommInitRank"));
    n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(sym("ncclCommDestroy"));
    n.send = reinterpret_cast<decltype(n.send)>(sym("ncclSend"));
    n.recv = reinterpret_cast<decltype(n.recv)>(sym("ncclRecv"));
    n.all_reduce = reinterpret_cast<decltype(n.all_reduce)>(sym("ncclAllReduce"));
    n.group_start = reinterpret_cast<decltype(n.group_start)>(sym("ncclGroupStart"));
    n.group_end = reinterpret_cast<decltype(n.group_end)>(sym("ncclGroupEnd"));
    n.error_string = reinterpret_cast<decltype(n.error_string)>(sym("ncclGetErrorString"));
    if (!n.get_unique_id || !n.comm_init_rank || !n.comm_destroy || !n.send || !n.recv || !n.all_reduce ||
        !n.group_start || !n.group_end || !n.error_string)
      failure = "libnccl.so.2 lacks a required symbol";
  });
  if (!failure.empty())
    throw Error(failure);
  return n;
}

void nccl_check(ncclResult_t r, const char *what) {
  if (r != ncclSuccess)
    throw Error(std::string(what) + ": " + nccl().error_string(r));
}

// ---------------- localisation kernels ----------------
__global__ void mark_foreign_senders(long long e0, long long e1, const int *sender, int o0, int o1, int *flag) {
  long long e = e0 + blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (e < e1) {
    int j = sender[e];
    if (j < o0 || j >= o1)
      flag[j] = 1;
  }
}
// Senders of edges [e0, e1) that this rank owns ([o0, o1)): flag[j - o0] = 1.
__global__ void mark_owned_senders(long long e0, long long e1, const int *sender, int o0, int o1, int *flag) {
  long long e = e0 + blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (e < e1) {
    int j = sender[e];
    if (j >= o0 && j < o1)
      flag[j - o0] = 1;
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
__global__ void compact(int n, const int *flag, const int *pos, int base, int *list) {
  int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j < n && flag[j])
    list[pos[j]] = j + base;
}
__global__ void local_offsets(int n_own, const int *row, int o0, int *out) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i <= n_own)
    out[i] = row[o0 + i] - row[o0];
}
__global__ void local_edges(long long e0, long long count, const int *sender, const int *reverse, int o0, int o1,
                            int n_own, const int *ghost_pos, int *lsender, int *lreverse) {
  long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (e >= count)
    return;
  int j = sender[e0 + e];
  lsender[e] = j >= o0 && j < o1 ? j - o0 : n_own + ghost_pos[j];
  long long r = reverse[e0 + e];
  lreverse[e] = r >= e0 && r < e0 + count ? int(r - e0) : -1;
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
} // namespace

std::string nccl_unique_id() {
  ncclUniqueId id;
  nccl_check(nccl().get_unique_id(&id), "ncclGetUniqueId");
  return std::string(id.internal, sizeof(id.internal));
}

struct Domain::Impl {
  int rank, world;
  ncclComm_t comm = nullptr;
  DeviceGeometry full{};
  bool localized = false;
  int n_own = 0, n_local = 0, o0 = 0, o1 = 0;
  std::vector<int> starts;                 // [world + 1] ownership ranges (internal ids)
  std::vector<int> send_count, ghost_off, ghost_count; // per peer
  std::vector<int *> send_list;            // per peer: local row ids to send (device)
};

Domain::Domain(int rank, int world, const void *unique_id) : impl_(std::make_unique<Impl>()) {
  if (world < 1 || rank < 0 || rank >= world || !unique_id)
    throw Error("Invalid domain rank or size");
  impl_->rank = rank;
  impl_->world = world;
  ncclUniqueId id;
  std::copy(static_cast<const char *>(unique_id), static_cast<const char *>(unique_id) + sizeof(id.internal),
            id.internal);
  nccl_check(nccl().comm_init_rank(&impl_->comm, world, id, rank), "ncclCommInitRank");
}
Domain::~Domain() {
  if (impl_ && impl_->comm)
    nccl().comm_destroy(impl_->comm);
}
int Domain::rank() const { return impl_->rank; }
int Domain::world() const { return impl_->world; }
int Domain::n_own() const { return impl_->n_own; }
int Domain::n_local() const { return impl_->n_local; }

void Domain::localize(Context &ctx) {
  auto &d = *impl_;
  const DeviceGeometry &g = ctx.geometry;
  d.full = g;
  int n = g.n, W = d.world;
  cudaStream_t s = ctx.stream;
  d.starts.assign(W + 1, 0);
  for (int r = 0; r <= W; ++r)
    d.starts[r] = int((long long)n * r / W);
  d.o0 = d.starts[d.rank];
  d.o1 = d.starts[d.rank + 1];
  d.n_own = d.o1 - d.o0;
  // Edge ranges of every rank's receivers (host copies of W + 1 row offsets).
  std::vector<int> edge_start(W + 1);
  for (int r = 0; r <= W; ++r)
    check(cudaMemcpyAsync(&edge_start[r], g.edge_offsets + d.starts[r], sizeof(int), cudaMemcpyDeviceToHost, s));
  check(cudaStreamSynchronize(s));
  long long E0 = edge_start[d.rank], E1 = edge_start[d.rank + 1];
  // Ghosts: foreign senders of this rank's edges, ascending internal id.
  int *flag = ctx.array<int>("domain.flag", size_t(n) + 1), *pos = ctx.array<int>("domain.pos", size_t(n) + 1);
  ctx.clear(flag, size_t(n + 1) * sizeof(int));
  if (E1 > E0)
    lapis::launch(mark_foreign_senders, blocks(E1 - E0), 256, 0, s, E0, E1, g.edge_sender, d.o0, d.o1, flag);
  lapis::launch(scan_flags, 1, 1024, 0, s, flag, pos, n);
  std::vector<int> pos_at(W + 1);
  for (int r = 0; r <= W; ++r)
    check(cudaMemcpyAsync(&pos_at[r], pos + d.starts[r], sizeof(int), cudaMemcpyDeviceToHost, s));
  check(cudaStreamSynchronize(s));
  int n_ghost = pos_at[W];
  d.n_local = d.n_own + n_ghost;
  int *ghosts = ctx.array<int>("domain.ghosts", std::max(n_ghost, 1));
  lapis::launch(compact, blocks(n), 256, 0, s, n, flag, pos, 0, ghosts);
  d.ghost_off.assign(W, 0);
  d.ghost_count.assign(W, 0);
  for (int r = 0; r < W; ++r) {
    d.ghost_off[r] = pos_at[r];
    d.ghost_count[r] = pos_at[r + 1] - pos_at[r];
  }
  // Send lists: this rank's atoms among each peer's senders.
  d.send_count.assign(W, 0);
  d.send_list.assign(W, nullptr);
  int *oflag = ctx.array<int>("domain.oflag", size_t(d.n_own) + 1), *opos = ctx.array<int>("domain.opos", size_t(d.n_own) + 1);
  for (int r = 0; r < W; ++r) {
    if (r == d.rank)
      continue;
    ctx.clear(oflag, size_t(d.n_own + 1) * sizeof(int));
    long long p0 = edge_start[r], p1 = edge_start[r + 1];
    if (p1 > p0)
      lapis::launch(mark_owned_senders, blocks(p1 - p0), 256, 0, s, p0, p1, g.edge_sender, d.o0, d.o1, oflag);
    lapis::launch(scan_flags, 1, 1024, 0, s, oflag, opos, d.n_own);
    int count = 0;
    check(cudaMemcpyAsync(&count, opos + d.n_own, sizeof(int), cudaMemcpyDeviceToHost, s));
    check(cudaStreamSynchronize(s));
    d.send_count[r] = count;
    d.send_list[r] = ctx.array<int>("domain.send." + std::to_string(r), std::max(count, 1));
    lapis::launch(compact, blocks(d.n_own), 256, 0, s, d.n_own, oflag, opos, 0, d.send_list[r]);
  }
  // The local graph: owned receivers, senders renumbered, a slice of the full edge list.
  long long El = E1 - E0;
  int *lrow = ctx.array<int>("domain.row", size_t(d.n_own) + 1);
  int *lsender = ctx.array<int>("domain.sender", size_t(std::max<long long>(El, 1)));
  int *lrev = ctx.array<int>("domain.reverse", size_t(std::max<long long>(El, 1)));
  int *lz = ctx.array<int>("domain.elements", std::max(d.n_local, 1));
  lapis::launch(local_offsets, blocks(d.n_own + 1), 256, 0, s, d.n_own, g.edge_offsets, d.o0, lrow);
  if (El)
    lapis::launch(local_edges, blocks(El), 256, 0, s, E0, El, g.edge_sender, g.edge_reverse, d.o0, d.o1, d.n_own,
                  pos, lsender, lrev);
  lapis::launch(local_elements, blocks(d.n_local), 256, 0, s, d.n_own, n_ghost, d.o0, g.elements, ghosts, lz);
  check(cudaGetLastError());
  DeviceGeometry l = g;
  l.n = d.n_own;
  l.elements = lz;
  l.edge_offsets = lrow;
  l.edge_sender = lsender;
  l.edge_shift = g.edge_shift + 3 * E0;
  l.edge_vector = g.edge_vector + E0;
  l.edge_r2 = g.edge_r2 + E0;
  l.edge_reverse = lrev;
  l.edge_capacity = El;
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
  const auto &N = nccl();
  cudaStream_t s = ctx.stream;
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
  nccl_check(N.group_start(), "ncclGroupStart");
  for (int r = 0; r < d.world; ++r) {
    if (r == d.rank)
      continue;
    if (d.send_count[r])
      nccl_check(N.send(sbuf[r], size_t(d.send_count[r]) * comps * width, ncclFloat32, r, d.comm, s), "ncclSend");
    if (d.ghost_count[r])
      nccl_check(N.recv(rbuf[r], size_t(d.ghost_count[r]) * comps * width, ncclFloat32, r, d.comm, s), "ncclRecv");
  }
  nccl_check(N.group_end(), "ncclGroupEnd");
  for (int r = 0; r < d.world; ++r)
    if (r != d.rank && d.ghost_count[r])
      lapis::launch(unpack_rows, blocks((long long)d.ghost_count[r] * comps * width), 256, 0, s, d.ghost_count[r], comps,
                    stride, width, static_cast<const int *>(nullptr), d.n_own + d.ghost_off[r], rbuf[r], x, 0);
}

void Domain::return_ghost_rows(Context &ctx, float *x, int comps, int stride, int width) {
  auto &d = *impl_;
  const auto &N = nccl();
  cudaStream_t s = ctx.stream;
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
  nccl_check(N.group_start(), "ncclGroupStart");
  for (int r = 0; r < d.world; ++r) {
    if (r == d.rank)
      continue;
    if (d.ghost_count[r])
      nccl_check(N.send(sbuf[r], size_t(d.ghost_count[r]) * comps * width, ncclFloat32, r, d.comm, s), "ncclSend");
    if (d.send_count[r])
      nccl_check(N.recv(rbuf[r], size_t(d.send_count[r]) * comps * width, ncclFloat32, r, d.comm, s), "ncclRecv");
  }
  nccl_check(N.group_end(), "ncclGroupEnd");
  // Added in rank order: a fixed order per atom.
  for (int r = 0; r < d.world; ++r)
    if (r != d.rank && d.send_count[r])
      lapis::launch(unpack_rows, blocks((long long)d.send_count[r] * comps * width), 256, 0, s, d.send_count[r], comps,
                    stride, width, static_cast<const int *>(d.send_list[r]), 0, rbuf[r], x, 1);
}

void Domain::gather_outputs(Context &ctx, const float *e, const float *f, const float *v, float *ef, float *ff,
                            float *vf) {
  auto &d = *impl_;
  cudaStream_t s = ctx.stream;
  int n = d.full.n;
  // ef, ff, vf are one contiguous [13 n] buffer: zero, place the owned rows, sum over ranks.
  ctx.clear(ef, size_t(n) * 13 * sizeof(float));
  if (d.n_own)
    lapis::launch(place_owned, blocks(d.n_own), 256, 0, s, d.n_own, d.o0, e, f, v, ef, ff, vf);
  if (d.world > 1)
    nccl_check(nccl().all_reduce(ef, ef, size_t(n) * 13, ncclFloat32, ncclSum, d.comm, s), "ncclAllReduce");
}
} // namespace lapis
