// Reader and writer of the reference's offline index formats.
//
//   <prefix>_node{s+1}_of{M}.dat   shard s: [u64 free_ptr | u64 medoid_ptr (shard 0)]
//                                  then fixed-size VamanaNode records
//                                  (src/vamana/vamana_node.hh:10-69,
//                                   tools/vamana_offline_builder.cc:1136-1213)
//   <prefix>.meta.json             dim, rabitq_bits, num_memory_nodes, rabitq_size, R, ...
//                                  (tools/vamana_offline_builder.cc:1245-1266)
//   <prefix>.rotation.bin          u32 dim | f32 P[dim*dim] col-major | f32 c'[dim] | f64 t_const
//                                  (tools/vamana_offline_builder.cc:1226-1243,
//                                   src/service/rabitq_artifacts.cc:22-73)
//
// A neighbour slot holds a RemotePtr (src/remote_pointer.hh:7-29):
// memory_node << 48 | byte_offset, 0 = null.  The reader maps every node to a
// dense slot g (g = k*M + s for the k-th node of shard s when the shards are the
// builder's round-robin split) and rewrites adjacency as slot indices.

#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <sstream>

#include "internal.h"

namespace dvs {

namespace {

thread_local std::string g_last_error;

bool read_file(const std::string& path, std::vector<uint8_t>& out) {
  std::ifstream in(path, std::ios::binary | std::ios::ate);
  if (!in.good()) return false;
  const std::streamsize sz = in.tellg();
  if (sz < 0) return false;
  in.seekg(0);
  out.resize(size_t(sz));
  if (sz > 0 && !in.read(reinterpret_cast<char*>(out.data()), sz)) return false;
  return true;
}

// Minimal JSON reader: flattens scalars to "a.b" -> text (strings unquoted).
class Json {
 public:
  explicit Json(const std::string& s) : s_(s) {}
  bool parse(std::map<std::string, std::string>& out) {
    pos_ = 0;
    ws();
    if (!value("", out)) return false;
    ws();
    return pos_ == s_.size();
  }

 private:
  void ws() {
    while (pos_ < s_.size() && std::isspace(static_cast<unsigned char>(s_[pos_]))) ++pos_;
  }
  bool str(std::string& o) {
    if (pos_ >= s_.size() || s_[pos_] != '"') return false;
    ++pos_;
    o.clear();
    while (pos_ < s_.size() && s_[pos_] != '"') {
      if (s_[pos_] == '\\' && pos_ + 1 < s_.size()) ++pos_;
      o.push_back(s_[pos_++]);
    }
    if (pos_ >= s_.size()) return false;
    ++pos_;
    return true;
  }
  bool value(const std::string& key, std::map<std::string, std::string>& out) {
    ws();
    if (pos_ >= s_.size()) return false;
    const char c = s_[pos_];
    if (c == '{') {
      ++pos_;
      ws();
      if (pos_ < s_.size() && s_[pos_] == '}') {
        ++pos_;
        return true;
      }
      for (;;) {
        ws();
        std::string k;
        if (!str(k)) return false;
        ws();
        if (pos_ >= s_.size() || s_[pos_] != ':') return false;
        ++pos_;
        if (!value(key.empty() ? k : key + "." + k, out)) return false;
        ws();
        if (pos_ < s_.size() && s_[pos_] == ',') {
          ++pos_;
          continue;
        }
        if (pos_ < s_.size() && s_[pos_] == '}') {
          ++pos_;
          return true;
        }
        return false;
      }
    }
    if (c == '[') {
      ++pos_;
      int depth = 1;
      while (pos_ < s_.size() && depth > 0) {
        if (s_[pos_] == '[') ++depth;
        if (s_[pos_] == ']') --depth;
        ++pos_;
      }
      return depth == 0;
    }
    if (c == '"') {
      std::string v;
      if (!str(v)) return false;
      out[key] = v;
      return true;
    }
    const size_t b = pos_;
    while (pos_ < s_.size() && s_[pos_] != ',' && s_[pos_] != '}' && s_[pos_] != ']' &&
           !std::isspace(static_cast<unsigned char>(s_[pos_])))
      ++pos_;
    if (pos_ == b) return false;
    out[key] = s_.substr(b, pos_ - b);
    return true;
  }
  const std::string& s_;
  size_t pos_ = 0;
};

bool get_u64(const std::map<std::string, std::string>& m, const std::string& k, uint64_t& v) {
  auto it = m.find(k);
  if (it == m.end()) return false;
  char* end = nullptr;
  const unsigned long long x = std::strtoull(it->second.c_str(), &end, 10);
  if (end == it->second.c_str() || *end != '\0') return false;
  v = x;
  return true;
}

std::string shard_path(const std::string& prefix, uint32_t s, uint32_t M) {
  return prefix + "_node" + std::to_string(s + 1) + "_of" + std::to_string(M) + ".dat";
}

}  // namespace

dvs_status fail(dvs_status s, const std::string& msg) {
  g_last_error = msg;
  return s;
}
void clear_error() { g_last_error.clear(); }
const std::string& last_error() { return g_last_error; }

dvs_status load_host_index(const std::string& prefix, HostIndex& out) {
  out = HostIndex{};
  if (prefix.empty()) return fail(DVS_ERR_ARG, "index prefix must not be empty");

  // ---- meta.json: load_artifacts (src/service/rabitq_artifacts.cc:22-40) ----
  std::vector<uint8_t> raw;
  const std::string meta_file = prefix + ".meta.json";
  if (!read_file(meta_file, raw)) return fail(DVS_ERR_IO, "missing metadata file: " + meta_file);
  std::map<std::string, std::string> meta;
  const std::string text(raw.begin(), raw.end());
  if (!Json(text).parse(meta)) return fail(DVS_ERR_FORMAT, "invalid metadata file " + meta_file + ": not JSON");
  uint64_t dim = 0, bits = 0, M = 0, rsize = 0, R = 0;
  for (auto [key, dst] : {std::pair<const char*, uint64_t*>{"dim", &dim}, {"rabitq_bits", &bits},
                          {"num_memory_nodes", &M}, {"rabitq_size", &rsize}, {"R", &R}}) {
    if (!get_u64(meta, key, *dst))
      return fail(DVS_ERR_FORMAT, "invalid metadata file " + meta_file + ": missing or non-integer \"" + key + "\"");
  }
  if (dim == 0 || dim > 65536) return fail(DVS_ERR_DIM, "metadata dim out of range: " + std::to_string(dim));
  if (bits != 1 && bits != 2 && bits != 4 && bits != 8)
    return fail(DVS_ERR_BITS, "rabitq_bits must be 1, 2, 4, or 8, got " + std::to_string(bits));
  if (M == 0 || M > 65535) return fail(DVS_ERR_FORMAT, "num_memory_nodes out of range: " + std::to_string(M));
  if (R == 0 || R > 255) return fail(DVS_ERR_FORMAT, "R out of range (edge_count is one byte): " + std::to_string(R));
  dvs_metric metric = DVS_METRIC_L2;
  if (auto it = meta.find("distance"); it != meta.end()) {
    if (it->second == "ip")
      metric = DVS_METRIC_IP;
    else if (it->second != "l2")
      return fail(DVS_ERR_FORMAT, "unknown distance \"" + it->second + "\" in " + meta_file);
  }

  // ---- rotation.bin (src/service/rabitq_artifacts.cc:42-71) ----
  const std::string rot_file = prefix + ".rotation.bin";
  if (!read_file(rot_file, raw)) return fail(DVS_ERR_IO, "missing RaBitQ rotation file: " + rot_file);
  if (raw.size() < 4) return fail(DVS_ERR_FORMAT, "failed to read rotation header: " + rot_file);
  uint32_t file_dim = 0;
  std::memcpy(&file_dim, raw.data(), 4);
  if (file_dim != dim)
    return fail(DVS_ERR_DIM, "rotation dim mismatch in " + rot_file + ": expected " + std::to_string(dim) +
                                 ", got " + std::to_string(file_dim));
  const size_t need = 4 + size_t(dim) * dim * 4 + size_t(dim) * 4 + 8;
  if (raw.size() < need) return fail(DVS_ERR_FORMAT, "failed to read complete RaBitQ payload: " + rot_file);
  out.rotation.resize(size_t(dim) * dim);
  out.rotated_centroid.resize(dim);
  std::memcpy(out.rotation.data(), raw.data() + 4, out.rotation.size() * 4);
  std::memcpy(out.rotated_centroid.data(), raw.data() + 4 + out.rotation.size() * 4, size_t(dim) * 4);
  double tc = 0.0;
  std::memcpy(&tc, raw.data() + 4 + out.rotation.size() * 4 + size_t(dim) * 4, 8);

  // sizes checked after the rotation file, in the reference's order
  // (rabitq_artifacts.cc:42-55, then compute_service.cc:562-568)
  NodeLayout lay{uint32_t(dim), uint32_t(R), uint32_t(bits)};
  if (rsize != lay.rabitq_size())
    return fail(DVS_ERR_FORMAT, "RaBitQ artifact size mismatch: expected " + std::to_string(lay.rabitq_size()) +
                                    ", got " + std::to_string(rsize));
  uint64_t node_size = 0;
  if (get_u64(meta, "node_size", node_size) && node_size != lay.node_size())
    return fail(DVS_ERR_FORMAT, "node_size mismatch: expected " + std::to_string(lay.node_size()) + ", got " +
                                    std::to_string(node_size));
  // ---- shards ----
  const size_t aligned = lay.aligned_size();
  std::vector<std::vector<uint8_t>> shards(M);
  std::vector<uint64_t> count(M);
  for (uint32_t s = 0; s < M; ++s) {
    const std::string f = shard_path(prefix, s, uint32_t(M));
    if (!read_file(f, shards[s])) return fail(DVS_ERR_IO, "missing shard file: " + f);
    if (shards[s].size() < 16) return fail(DVS_ERR_FORMAT, "shard shorter than its 16-byte header: " + f);
    uint64_t free_ptr = 0;
    std::memcpy(&free_ptr, shards[s].data(), 8);
    if (free_ptr < 16 || free_ptr > shards[s].size() || (free_ptr - 16) % aligned != 0)
      return fail(DVS_ERR_FORMAT, "shard free pointer " + std::to_string(free_ptr) + " does not end a node in " + f);
    count[s] = (free_ptr - 16) / aligned;
  }
  uint64_t n = 0, max_count = 0;
  for (uint32_t s = 0; s < M; ++s) {
    n += count[s];
    max_count = std::max(max_count, count[s]);
  }
  if (n == 0) return fail(DVS_ERR_FORMAT, "index holds no nodes");
  if (n >= kEmpty) return fail(DVS_ERR_FORMAT, "index holds too many nodes");
  // dense slots: k-major, then shard
  std::vector<std::vector<uint32_t>> slot(M);
  {
    uint32_t g = 0;
    for (uint32_t s = 0; s < M; ++s) slot[s].resize(count[s]);
    for (uint64_t k = 0; k < max_count; ++k)
      for (uint32_t s = 0; s < M; ++s)
        if (k < count[s]) slot[s][k] = g++;
  }
  auto resolve = [&](uint64_t raw_ptr, uint32_t& g) -> bool {
    const uint64_t s = raw_ptr >> 48, off = raw_ptr & ((uint64_t(1) << 48) - 1);
    if (s >= M || off < 16 || (off - 16) % aligned != 0) return false;
    const uint64_t k = (off - 16) / aligned;
    if (k >= count[s]) return false;
    g = slot[s][k];
    return true;
  };
  out.adj.assign(n * R, kEmpty);
  out.records.resize(n * rsize);
  out.vecs.resize(n * dim);
  out.ids.resize(n);
  for (uint32_t s = 0; s < M; ++s) {
    for (uint64_t k = 0; k < count[s]; ++k) {
      const uint8_t* node = shards[s].data() + 16 + k * aligned;
      const uint32_t g = slot[s][k];
      std::memcpy(&out.ids[g], node + lay.off_id(), 4);
      const uint8_t ec = node[lay.off_edge_count()];
      if (ec > R)
        return fail(DVS_ERR_FORMAT, "node " + std::to_string(out.ids[g]) + " has edge_count " + std::to_string(ec) +
                                        " > R " + std::to_string(R));
      std::memcpy(&out.vecs[size_t(g) * dim], node + lay.off_vector(), size_t(dim) * 4);
      std::memcpy(&out.records[size_t(g) * rsize], node + lay.off_rabitq(), rsize);
      // neighbours: the first edge_count slots, nulls skipped (src/vamana/vamana.hh:175-178)
      uint32_t w = 0;
      for (uint32_t j = 0; j < ec; ++j) {
        uint64_t p = 0;
        std::memcpy(&p, node + lay.off_neighbors() + size_t(j) * 8, 8);
        if (p == 0) continue;
        uint32_t t = 0;
        if (!resolve(p, t))
          return fail(DVS_ERR_FORMAT, "node " + std::to_string(out.ids[g]) + " has a neighbour pointer outside the shards");
        out.adj[size_t(g) * R + w++] = t;
      }
    }
  }
  uint64_t mp = 0;
  std::memcpy(&mp, shards[0].data() + 8, 8);
  uint32_t medoid = 0;
  if (mp == 0 || !resolve(mp, medoid)) return fail(DVS_ERR_FORMAT, "medoid pointer of shard 1 does not name a node");

  for (size_t i = 0; i < out.vecs.size(); ++i)
    if (!std::isfinite(out.vecs[i])) return fail(DVS_ERR_FORMAT, "index vectors contain a non-finite value");

  dvs_index_info& info = out.info;
  info.num_vectors = n;
  info.dim = uint32_t(dim);
  info.R = uint32_t(R);
  info.rabitq_bits = uint32_t(bits);
  info.rabitq_size = uint32_t(rsize);
  info.num_memory_nodes = uint32_t(M);
  info.medoid = medoid;
  info.metric = metric;
  info.t_const = tc;
  return DVS_OK;
}

}  // namespace dvs

using dvs::fail;

extern "C" {

const char* dvs_last_error(void) { return dvs::last_error().c_str(); }

const char* dvs_status_string(dvs_status s) {
  switch (s) {
    case DVS_OK: return "ok";
    case DVS_ERR_ARG: return "invalid argument";
    case DVS_ERR_IO: return "i/o error";
    case DVS_ERR_FORMAT: return "malformed index file";
    case DVS_ERR_DIM: return "dimension mismatch";
    case DVS_ERR_BITS: return "unsupported RaBitQ bit width";
    case DVS_ERR_CUDA: return "CUDA error";
    case DVS_ERR_PEER: return "peer access unavailable";
    case DVS_ERR_HOP_LIMIT: return "expansion limit reached";
    case DVS_ERR_TIMEOUT: return "device wait timed out";
    case DVS_ERR_OOM: return "out of memory";
    case DVS_ERR_CAPACITY: return "capacity exceeded";
    case DVS_ERR_UNSUPPORTED: return "unsupported";
    case DVS_ERR_NO_DEVICE: return "no CUDA device";
  }
  return "unknown status";
}

struct dvs_host_index {
  dvs::HostIndex h;
};

dvs_status dvs_host_index_load(const char* index_prefix, dvs_host_index** out) {
  if (!index_prefix || !out) return fail(DVS_ERR_ARG, "null argument");
  *out = nullptr;
  auto* h = new (std::nothrow) dvs_host_index;
  if (!h) return fail(DVS_ERR_OOM, "host allocation failed");
  const dvs_status s = dvs::load_host_index(index_prefix, h->h);
  if (s != DVS_OK) {
    delete h;
    return s;
  }
  *out = h;
  return DVS_OK;
}

dvs_status dvs_host_index_info(const dvs_host_index* h, dvs_index_info* out) {
  if (!h || !out) return fail(DVS_ERR_ARG, "null argument");
  *out = h->h.info;
  return DVS_OK;
}

dvs_status dvs_host_index_arrays(const dvs_host_index* h, const uint32_t** adj, const uint8_t** records,
                                 const float** vecs, const uint32_t** ids, const float** rotation,
                                 const float** rotated_centroid) {
  if (!h) return fail(DVS_ERR_ARG, "null index");
  if (adj) *adj = h->h.adj.data();
  if (records) *records = h->h.records.data();
  if (vecs) *vecs = h->h.vecs.data();
  if (ids) *ids = h->h.ids.data();
  if (rotation) *rotation = h->h.rotation.data();
  if (rotated_centroid) *rotated_centroid = h->h.rotated_centroid.data();
  return DVS_OK;
}

void dvs_host_index_free(dvs_host_index* h) { delete h; }

dvs_status dvs_write_index(const dvs_write_params* p, const float* h_vecs, const uint32_t* h_adj,
                           const uint8_t* h_records, const float* h_rotation, const float* h_rotated_centroid,
                           const uint32_t* h_ids) {
  if (!p || !p->index_prefix || !h_vecs || !h_adj || !h_records || !h_rotation || !h_rotated_centroid)
    return fail(DVS_ERR_ARG, "null argument");
  const uint64_t n = p->num_vectors;
  const uint32_t M = p->num_memory_nodes;
  if (n == 0 || n >= dvs::kEmpty) return fail(DVS_ERR_ARG, "num_vectors out of range");
  if (M == 0 || M > 65535) return fail(DVS_ERR_ARG, "num_memory_nodes out of range");
  if (p->R == 0 || p->R > 255) return fail(DVS_ERR_ARG, "R out of range");
  if (p->rabitq_bits != 1 && p->rabitq_bits != 2 && p->rabitq_bits != 4 && p->rabitq_bits != 8)
    return fail(DVS_ERR_BITS, "rabitq_bits must be 1, 2, 4, or 8");
  if (p->medoid >= n) return fail(DVS_ERR_ARG, "medoid out of range");
  dvs::NodeLayout lay{p->dim, p->R, p->rabitq_bits};
  const size_t aligned = lay.aligned_size(), rs = lay.rabitq_size();
  auto rptr = [&](uint64_t i) -> uint64_t { return (uint64_t(i % M) << 48) | (16 + (i / M) * aligned); };
  const std::string prefix(p->index_prefix);
  for (uint32_t s = 0; s < M; ++s) {
    const uint64_t cnt = n / M + (s < n % M ? 1 : 0);
    std::vector<uint8_t> buf(16 + cnt * aligned, 0);
    const uint64_t sz = buf.size();
    std::memcpy(buf.data(), &sz, 8);
    if (s == 0) {
      const uint64_t mp = rptr(p->medoid);
      std::memcpy(buf.data() + 8, &mp, 8);
    }
    for (uint64_t k = 0; k < cnt; ++k) {
      const uint64_t i = k * M + s;
      uint8_t* node = buf.data() + 16 + k * aligned;
      const uint64_t header = (i == p->medoid) ? (uint64_t(1) << 16) : 0;  // HEADER_IS_MEDOID
      std::memcpy(node, &header, 8);
      const uint32_t id = h_ids ? h_ids[i] : uint32_t(i);
      std::memcpy(node + lay.off_id(), &id, 4);
      std::memcpy(node + lay.off_vector(), h_vecs + i * p->dim, size_t(p->dim) * 4);
      std::memcpy(node + lay.off_rabitq(), h_records + i * rs, rs);
      uint8_t ec = 0;
      for (uint32_t j = 0; j < p->R; ++j) {
        const uint32_t t = h_adj[i * p->R + j];
        if (t == dvs::kEmpty) continue;
        if (t >= n) return fail(DVS_ERR_ARG, "adjacency entry out of range");
        const uint64_t q = rptr(t);
        std::memcpy(node + lay.off_neighbors() + size_t(ec) * 8, &q, 8);
        ++ec;
      }
      node[lay.off_edge_count()] = ec;
    }
    const std::string f = dvs::shard_path(prefix, s, M);
    std::ofstream o(f, std::ios::binary);
    if (!o.good()) return fail(DVS_ERR_IO, "failed to open output shard file: " + f);
    o.write(reinterpret_cast<const char*>(buf.data()), std::streamsize(buf.size()));
    if (!o.good()) return fail(DVS_ERR_IO, "failed to write output shard file: " + f);
  }
  {
    const std::string f = prefix + ".rotation.bin";
    std::ofstream o(f, std::ios::binary);
    if (!o.good()) return fail(DVS_ERR_IO, "failed to open rotation matrix file: " + f);
    const uint32_t d = p->dim;
    o.write(reinterpret_cast<const char*>(&d), 4);
    o.write(reinterpret_cast<const char*>(h_rotation), std::streamsize(size_t(d) * d * 4));
    o.write(reinterpret_cast<const char*>(h_rotated_centroid), std::streamsize(size_t(d) * 4));
    o.write(reinterpret_cast<const char*>(&p->t_const), 8);
    if (!o.good()) return fail(DVS_ERR_IO, "failed to write rotation matrix file: " + f);
  }
  {
    const std::string f = prefix + ".meta.json";
    std::ofstream o(f);
    if (!o.good()) return fail(DVS_ERR_IO, "failed to open metadata file: " + f);
    const uint64_t mp = rptr(p->medoid);
    char alpha[64];
    std::snprintf(alpha, sizeof(alpha), "%.15g", p->alpha);
    o << "{\n  \"R\": " << p->R << ",\n  \"alpha\": " << alpha << ",\n  \"beam_width\": " << p->beam_width
      << ",\n  \"beam_width_construction\": " << p->beam_width << ",\n  \"data_file\": \"synthetic\",\n  \"dim\": "
      << p->dim << ",\n  \"distance\": \"" << (p->metric == DVS_METRIC_IP ? "ip" : "l2")
      << "\",\n  \"medoid\": {\n    \"memory_node\": " << (mp >> 48) << ",\n    \"offset\": "
      << (mp & ((uint64_t(1) << 48) - 1)) << "\n  },\n  \"node_size\": " << lay.node_size()
      << ",\n  \"num_memory_nodes\": " << M << ",\n  \"num_vectors\": " << n << ",\n  \"output_prefix\": \""
      << prefix << "\",\n  \"rabitq_bits\": " << p->rabitq_bits << ",\n  \"rabitq_size\": " << rs << "\n}\n";
    if (!o.good()) return fail(DVS_ERR_IO, "failed to write metadata file: " + f);
  }
  return DVS_OK;
}

}  // extern "C"
