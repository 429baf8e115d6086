// Host form of the domain-decomposition exchange plan (the rules Domain::localize applies on
// the device with its plan kernels), for checks without a GPU.
//
// Atoms have ids 0..n-1; rank r of W owns ids [n r / W, n (r + 1) / W).  From this rank's
// CSR rows (its receivers, in id order, each listing the sender id of every edge):
//   ghosts      the senders the rank does not own, ascending id; those owned by peer q form
//               one contiguous block (ghost_counts[q] of them);
//   sends to q  the rank's receivers with at least one edge from an atom of q, ascending
//               (send_counts[q] of them), as global ids.
// With a symmetric edge relation, rank r's sends to q equal q's ghost block from r, element
// for element: the owner ships exactly the rows its peer needs, in the order the peer
// stores them, without requests.
#include "mace/c_api.h"
#include <algorithm>
#include <stdexcept>
#include <string>
#include <vector>

namespace lapis {
void set_c_api_error(const std::string &message);
}

int lapis_exchange_plan_host(int n, int rank, int world, const int *row, const int *sender, int *send_counts,
                             int *ghost_counts, int *ghosts, int *sends, long long capacity) {
  try {
    lapis::set_c_api_error("");
    if (n < 0 || world < 1 || rank < 0 || rank >= world || !send_counts || !ghost_counts)
      throw std::runtime_error("Invalid exchange-plan arguments");
    std::vector<long long> start(world + 1);
    for (int r = 0; r <= world; ++r)
      start[r] = (long long)n * r / world;
    const long long o0 = start[rank], o1 = start[rank + 1], own = o1 - o0;
    if (own && (!row || !sender))
      throw std::runtime_error("Null exchange-plan rows");
    auto owner = [&](int j) { return int(std::upper_bound(start.begin(), start.end(), (long long)j) - start.begin()) - 1; };
    std::vector<char> foreign(size_t(n), 0);
    std::vector<std::vector<int>> to(world);
    for (long long w = 0; w < own; ++w) {
      std::vector<char> seen(size_t(world), 0);
      for (int e = row[w]; e < row[w + 1]; ++e) {
        int j = sender[e];
        if (j < 0 || j >= n)
          throw std::runtime_error("Sender id out of range");
        int q = owner(j);
        if (q == rank)
          continue;
        foreign[size_t(j)] = 1;
        if (!seen[size_t(q)]) {
          seen[size_t(q)] = 1;
          to[size_t(q)].push_back(int(o0 + w));
        }
      }
    }
    std::vector<int> ghost;
    for (int j = 0; j < n; ++j)
      if (foreign[size_t(j)])
        ghost.push_back(j);
    std::vector<int> send;
    for (int q = 0; q < world; ++q) {
      ghost_counts[q] = int(std::count_if(ghost.begin(), ghost.end(), [&](int j) { return owner(j) == q; }));
      send_counts[q] = int(to[size_t(q)].size());
      send.insert(send.end(), to[size_t(q)].begin(), to[size_t(q)].end());
    }
    if (capacity >= (long long)std::max(ghost.size(), send.size())) {
      if (ghosts)
        std::copy(ghost.begin(), ghost.end(), ghosts);
      if (sends)
        std::copy(send.begin(), send.end(), sends);
    }
    return 0;
  } catch (const std::exception &e) {
    lapis::set_c_api_error(e.what());
    return -1;
  }
}
