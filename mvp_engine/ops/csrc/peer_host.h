// Host side of the peer-memory copy that rides along compute kernels (PeerPull in common.cuh).
#pragma once

#include <cstdint>
#include <vector>

#include <c10/util/Optional.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include "common.cuh"

namespace mvp {

// Grid rows a compute kernel adds for the copy: at 64+ copy CTAs of 320 threads, 8 loads in flight
// each, ~3 MB is outstanding, enough to keep one NVLink direction busy.
constexpr int kPullRows = 1;

// pull = [src, dst, bytes, ready_slot, seq, timeout_ns] (device addresses as integers); empty: no copy.
inline PeerPull make_peer_pull(const c10::optional<std::vector<int64_t>>& pull) {
  PeerPull j{};
  if (!pull.has_value() || pull->empty()) return j;
  const auto& v = *pull;
  TORCH_CHECK(v.size() == 6, "pull = [src, dst, bytes, ready_slot, seq, timeout_ns]");
  TORCH_CHECK(v[0] != 0 && v[1] != 0 && v[3] != 0, "pull: null address");
  TORCH_CHECK(v[0] % 16 == 0 && v[1] % 16 == 0 && v[2] % 16 == 0, "pull: 16-byte aligned addresses and size");
  TORCH_CHECK(v[3] % 8 == 0, "pull: 8-byte aligned ready slot");
  TORCH_CHECK(v[5] > 0, "pull: the wait for the owner needs a positive bound");
  j.src = reinterpret_cast<const uint4*>(v[0]);
  j.dst = reinterpret_cast<uint4*>(v[1]);
  j.n16 = v[2] / 16;
  j.ready = reinterpret_cast<const unsigned long long*>(v[3]);
  j.seq = static_cast<unsigned long long>(v[4]);
  j.timeout_ns = static_cast<unsigned long long>(v[5]);
  j.rows = j.n16 > 0 ? kPullRows : 0;
  return j;
}

// route = [world, rank, chunk, ld, col0, col0_k, dst_0 .. dst_{world-1}]; empty: no routing.
inline UlyssesRoute make_ulysses_route(const c10::optional<std::vector<int64_t>>& route) {
  UlyssesRoute u{};
  if (!route.has_value() || route->empty()) return u;
  const auto& v = *route;
  TORCH_CHECK(v.size() >= 7, "route = [world, rank, chunk, ld, col0, col0_k, dst...]");
  u.world = static_cast<int>(v[0]);
  u.rank = static_cast<int>(v[1]);
  u.chunk = static_cast<int>(v[2]);
  u.ld = v[3];
  u.col0 = static_cast<int>(v[4]);
  u.col0_k = static_cast<int>(v[5]);
  TORCH_CHECK(u.world >= 1 && u.world <= 8 && static_cast<int>(v.size()) == 6 + u.world,
              "route: 1..8 ranks, one destination each");
  TORCH_CHECK(u.rank >= 0 && u.rank < u.world && u.chunk > 0, "route: rank / chunk");
  TORCH_CHECK(u.ld % 8 == 0 && u.col0 % 8 == 0 && u.col0_k % 8 == 0, "route: 16-byte aligned rows and columns");
  for (int j = 0; j < u.world; ++j) {
    TORCH_CHECK(v[6 + j] != 0 && v[6 + j] % 16 == 0, "route: 16-byte aligned destinations");
    u.dst[j] = reinterpret_cast<void*>(v[6 + j]);
  }
  return u;
}

// Stand-alone launch of the same copy (used when the compute kernel has no tiles to run).
void launch_peer_pull(const PeerPull& j, int* status, cudaStream_t stream);

}  // namespace mvp
