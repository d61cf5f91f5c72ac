/* C++ host side of the query path: ComputeService over the C ABI of
 * dvs_b200.h.
 *
 * It keeps the reference service's interface for this path
 * (src/service/compute_service.hh:63-103): the search-mode / beam-width / k
 * configuration and its defaults and checks (src/common/configuration.hh:87-205),
 * search / insert / load_index / store_index / status with the same argument
 * meaning, results truncated to k (compute_service.cc:215-217), and the same
 * errors: a query or vector of the wrong dimension throws
 * std::invalid_argument("search dimension mismatch" / "insert dimension
 * mismatch"), load_index / store_index return false and fill *error_message.
 * Where the reference prints an option error and exits
 * (validate_compute_node_options), this throws dvs::ConfigError with the same
 * message.  The index lives in HBM, so the RDMA transport, CPU caches, routing
 * and worker/coroutine options have nothing to configure and are not here.
 *
 * Header-only: include it and link libdvs_b200.so (the C ABI stays the
 * boundary; no C++ types cross it).
 */
#pragma once

#include <algorithm>
#include <cctype>
#include <cstdint>
#include <mutex>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "dvs_b200.h"

namespace dvs {

/* An option error of validate_compute_node_options (configuration.hh:152-198). */
class ConfigError : public std::invalid_argument {
 public:
  using std::invalid_argument::invalid_argument;
};

/* A failing call of the C ABI: the status and dvs_last_error(). */
class Error : public std::runtime_error {
 public:
  Error(dvs_status s, const std::string& what) : std::runtime_error(what), status(s) {}
  dvs_status status;
};

inline void check(dvs_status s) {
  if (s != DVS_OK) throw Error(s, dvs_last_error());
}

/* The query-path options of IndexConfiguration (configuration.hh:87-154), with
 * the reference's names and defaults. */
struct Configuration {
  std::string data_path;               /* --data-path */
  std::string index_prefix;            /* --index-prefix */
  bool load_index = false;             /* --load-index: open the index at start-up */
  bool store_index = false;            /* --store-index */
  bool ip_dist = false;                /* --ip-dist (the metric is the index's own) */
  uint32_t beam_width = 0;             /* --beam-width / --ef-search, required */
  uint32_t beam_width_construction = 200; /* --beam-width-construction / --ef-construction */
  uint32_t k = 0;                      /* --k, required */
  uint32_t R = 64;                     /* --R / -m */
  float alpha = 1.2f;                  /* --alpha */
  uint32_t rabitq_bits = 1;            /* --rabitq-bits */
  std::string search_mode = "exact_gpu"; /* --search-mode: exact_gpu | rabitq_gpu */
  int gpu_device = 0;                  /* --gpu-device */
  uint32_t dim = 0;                    /* --dim, required */
  /* Beyond the reference's options: several devices hold one replica each
   * (or, with shard = true, one memory-node shard each); empty = {gpu_device}. */
  std::vector<int> gpu_devices;
  bool shard = false;

  /* normalize_search_mode (configuration.hh:200-205). */
  static std::string normalize_search_mode(std::string value) {
    std::transform(value.begin(), value.end(), value.begin(),
                   [](unsigned char ch) { return static_cast<char>(std::tolower(ch)); });
    return value;
  }

  bool use_rabitq_search() const { return search_mode == "rabitq_gpu"; }

  /* The checks of validate_compute_node_options that concern this path
   * (the worker thread count is not required: no CPU workers run queries). */
  void validate() {
    search_mode = normalize_search_mode(search_mode);
    if (beam_width == 0 || k == 0 || dim == 0)
      throw ConfigError("Parameters beam-width (ef-search), k, and dim are required");
    if (store_index && load_index)
      throw ConfigError("--store-index and --load-index cannot be used in conjunction");
    if ((store_index || load_index) && index_prefix.empty() && data_path.empty())
      throw ConfigError("--data-path or --index-prefix is required when --load-index or --store-index is set");
    if (search_mode != "exact_gpu" && search_mode != "rabitq_gpu")
      throw ConfigError("--search-mode must be exact_gpu or rabitq_gpu");
    if (rabitq_bits != 1 && rabitq_bits != 2 && rabitq_bits != 4 && rabitq_bits != 8)
      throw ConfigError("--rabitq-bits must be 1, 2, 4, or 8");
    if (beam_width < k) throw ConfigError("beam_width must be >= k"); /* vamana.hh:49 */
  }

  /* index_path::resolve_prefix (src/common/index_path.hh:19-24). */
  std::string resolved_index_prefix() const {
    if (!index_prefix.empty()) return index_prefix;
    if (data_path.empty()) throw ConfigError("data path must not be empty");
    std::string base = data_path;
    const size_t slash = base.find_last_of('/');
    const size_t dot = base.find_last_of('.');
    if (dot != std::string::npos && (slash == std::string::npos || dot > slash))
      base = slash == std::string::npos ? std::string(".") : base.substr(0, slash);
    return base + "/dump/index_m" + std::to_string(R) + "_efc" + std::to_string(beam_width_construction);
  }
};

class ComputeService {
 public:
  struct InsertItem {
    uint32_t id;
    std::vector<float> values;
  };

  struct Status {
    std::string state{"running"};
    size_t vectors_inserted{};
    uint32_t dimension{};
    uint32_t threads{};
  };

  /* Per-operation counters the GPU path produces: the device-side
   * counterparts of statistics::ThreadStatistics (src/common/statistics.hh:188-251). */
  struct Statistics {
    uint64_t processed_queries{}, processed_inserts{};
    uint64_t visited_neighborlists{}, query_distcomps{}, query_exact_reranks{};
    uint64_t build_distcomps{}, build_overflow_prunes{};
    double query_device_ms{}, insert_device_ms{};
  };

  explicit ComputeService(const Configuration& config) : config_(config) {
    config_.validate();
    if (config_.load_index) {
      std::string msg;
      if (!load_index(config_.resolved_index_prefix(), &msg)) throw ConfigError(msg);
    }
  }
  ~ComputeService() {
    if (index_) dvs_close(index_);
  }
  ComputeService(const ComputeService&) = delete;
  ComputeService& operator=(const ComputeService&) = delete;

  /* ComputeService::insert (compute_service.cc:152-196): every item must have
   * `dim` values; returns the number inserted. */
  size_t insert(const std::vector<InsertItem>& batch) {
    if (batch.empty()) return 0;
    std::vector<float> vectors;
    std::vector<uint32_t> ids;
    vectors.reserve(batch.size() * size_t(config_.dim));
    ids.reserve(batch.size());
    for (const auto& item : batch) {
      if (item.values.size() != config_.dim) throw std::invalid_argument("insert dimension mismatch");
      vectors.insert(vectors.end(), item.values.begin(), item.values.end());
      ids.push_back(item.id);
    }
    std::lock_guard<std::mutex> g(mu_);
    require_index();
    dvs_insert_params p{};
    p.beam_width_construction = config_.beam_width_construction;
    p.alpha = config_.alpha;
    dvs_insert_stats st{};
    check(dvs_insert(index_, vectors.data(), ids.data(), uint32_t(batch.size()), config_.dim, &p, &st));
    vectors_inserted_ += st.inserted;
    stats_.processed_inserts += st.inserted;
    stats_.build_distcomps += st.distances;
    stats_.visited_neighborlists += st.expansions;
    stats_.build_overflow_prunes += st.full_prunes;
    stats_.insert_device_ms += double(st.device_ms) + st.prune_ms + st.reverse_ms;
    return size_t(st.inserted);
  }

  /* ComputeService::search (compute_service.cc:193-227): the top
   * min(k, --k) node ids of one query, nearest first. */
  std::vector<uint32_t> search(const std::vector<float>& query, uint32_t k) {
    if (query.size() != config_.dim) throw std::invalid_argument("search dimension mismatch");
    std::vector<std::vector<uint32_t>> r = search_batch(query.data(), 1, k);
    return std::move(r[0]);
  }

  /* A batch of nq queries (nq * dim floats) in one device launch. */
  std::vector<std::vector<uint32_t>> search_batch(const float* queries, size_t nq, uint32_t k) {
    std::vector<std::vector<uint32_t>> out(nq);
    if (nq == 0) return out;
    const uint32_t kk = std::min(k, config_.k);
    std::vector<uint32_t> ids(nq * size_t(kk));
    std::vector<float> dist(nq * size_t(kk));
    dvs_stats st{};
    {
      std::lock_guard<std::mutex> g(mu_);
      require_index();
      check(dvs_search(index_, queries, uint32_t(nq), config_.dim, kk, config_.beam_width, mode(), ids.data(),
                       dist.data(), &st));
      stats_.processed_queries += nq;
      stats_.visited_neighborlists += st.expansions;
      stats_.query_distcomps += st.estimates;
      stats_.query_exact_reranks += st.reranked;
      stats_.query_device_ms += st.device_ms;
    }
    for (size_t q = 0; q < nq; ++q) {
      for (uint32_t j = 0; j < kk; ++j) {
        const uint32_t id = ids[q * kk + j];
        if (id != 0xFFFFFFFFu) out[q].push_back(id);  /* fewer than k reachable */
      }
    }
    return out;
  }

  /* load_index + maybe_load_rabitq_artifacts (compute_service.cc:280-310,
   * 520-593): in rabitq_gpu mode the artifacts' dim and bits must match the
   * options. */
  bool load_index(const std::string& path, std::string* error_message = nullptr) {
    std::vector<int> devs = config_.gpu_devices.empty() ? std::vector<int>{config_.gpu_device} : config_.gpu_devices;
    dvs_open_params p{};
    p.index_prefix = path.c_str();
    p.devices = devs.data();
    p.num_devices = uint32_t(devs.size());
    p.placement = config_.shard ? DVS_PLACE_SHARD : DVS_PLACE_REPLICATE;
    p.expect_dim = config_.use_rabitq_search() ? config_.dim : 0;
    p.expect_bits = config_.use_rabitq_search() ? config_.rabitq_bits : 0;
    dvs_index* ix = nullptr;
    if (dvs_open(&p, &ix) != DVS_OK) {
      if (error_message) *error_message = dvs_last_error();
      return false;
    }
    dvs_index_info info{};
    dvs_index_get_info(ix, &info);
    if (info.dim != config_.dim) {
      dvs_close(ix);
      if (error_message)
        *error_message = "search dimension mismatch: index " + std::to_string(info.dim) + ", --dim " +
                         std::to_string(config_.dim);
      return false;
    }
    std::lock_guard<std::mutex> g(mu_);
    if (index_) dvs_close(index_);
    index_ = ix;
    return true;
  }

  /* store_index (compute_service.cc:321-337): the index as it is now, inserts
   * included, in the shard/meta/rotation formats with num_memory_nodes shards. */
  bool store_index(const std::string& path, std::string* error_message = nullptr, uint32_t num_memory_nodes = 1) {
    std::lock_guard<std::mutex> g(mu_);
    if (!index_) {
      if (error_message) *error_message = "no index loaded";
      return false;
    }
    dvs_index_info info{};
    dvs_index_get_info(index_, &info);
    const size_t n = size_t(info.num_vectors), d = info.dim;
    std::vector<uint32_t> adj(n * info.R), ids(n);
    std::vector<uint8_t> records(n * info.rabitq_size);
    std::vector<float> vecs(n * d), P(d * d), c_rot(d);
    dvs_write_params w{};
    w.index_prefix = path.c_str();
    w.num_vectors = info.num_vectors;
    w.dim = info.dim;
    w.R = info.R;
    w.rabitq_bits = info.rabitq_bits;
    w.num_memory_nodes = num_memory_nodes;
    w.medoid = info.medoid;
    w.beam_width = config_.beam_width_construction;
    w.alpha = config_.alpha;
    w.metric = info.metric;
    w.t_const = info.t_const;
    if (dvs_index_download(index_, adj.data(), records.data(), vecs.data(), ids.data()) != DVS_OK ||
        dvs_index_artifacts(index_, P.data(), c_rot.data()) != DVS_OK ||
        dvs_write_index(&w, vecs.data(), adj.data(), records.data(), P.data(), c_rot.data(), ids.data()) != DVS_OK) {
      if (error_message) *error_message = dvs_last_error();
      return false;
    }
    return true;
  }

  /* ComputeService::status (compute_service.cc:339-347); no CPU worker threads. */
  Status status() const { return {"running", size_t(vectors_inserted_), config_.dim, 0}; }

  Statistics statistics() const {
    std::lock_guard<std::mutex> g(mu_);
    return stats_;
  }
  void clear_thread_statistics() {
    std::lock_guard<std::mutex> g(mu_);
    stats_ = Statistics{};
  }

  const Configuration& config() const { return config_; }
  /* The open index, for the rest of the C ABI (device searches, timing). */
  dvs_index* index() const { return index_; }

 private:
  dvs_mode mode() const { return config_.use_rabitq_search() ? DVS_MODE_RABITQ_GPU : DVS_MODE_EXACT_GPU; }
  void require_index() const {
    if (!index_) throw Error(DVS_ERR_ARG, "no index loaded");
  }

  Configuration config_;
  dvs_index* index_ = nullptr;
  uint64_t vectors_inserted_ = 0;
  Statistics stats_;
  mutable std::mutex mu_;
};

}  // namespace dvs
