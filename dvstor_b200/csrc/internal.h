// Internal declarations shared by the host-side translation units.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "dvs_b200.h"

namespace dvs {

constexpr uint32_t kEmpty = 0xFFFFFFFFu;
constexpr uint32_t kBeamSlack = 64;  // kRabitqSearchBeamSlack, src/vamana/vamana.hh:33

// Thread-local last error; returns `s` so callers can `return fail(...)`.
dvs_status fail(dvs_status s, const std::string& msg);
void clear_error();

// Sizes of the VamanaNode record (src/vamana/vamana_node.hh:10-69).
struct NodeLayout {
  uint32_t dim = 0, R = 0, bits = 0;
  uint32_t rabitq_size() const { return (bits * dim + 7) / 8 + 8; }
  uint32_t packed() const { return (bits * dim + 7) / 8; }
  size_t off_id() const { return 8; }
  size_t off_edge_count() const { return 12; }
  size_t off_vector() const { return 16; }
  size_t off_rabitq() const { return 16 + size_t(dim) * 4; }
  size_t off_neighbors() const { return off_rabitq() + rabitq_size(); }
  size_t node_size() const { return off_neighbors() + size_t(R) * 8; }
  size_t aligned_size() const { return (node_size() + 7) & ~size_t(7); }
};

// An index in host memory, dense slot order (slot g = k*M + s).
struct HostIndex {
  dvs_index_info info{};
  std::vector<uint32_t> adj;       // n*R slots, kEmpty fill, non-empty first
  std::vector<uint8_t> records;    // n*rabitq_size, reference record layout
  std::vector<float> vecs;         // n*dim
  std::vector<uint32_t> ids;       // stored node ids
  std::vector<float> rotation;     // dim*dim column-major
  std::vector<float> rotated_centroid;
};

dvs_status load_host_index(const std::string& prefix, HostIndex& out);

}  // namespace dvs
