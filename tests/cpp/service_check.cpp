// Drives the C++ host side (include/dvs_b200_service.hpp) for the tests.
//
//   service_check config
//       option checks and errors that need no GPU; prints one line per check
//   service_check search <prefix> <dim> <k> <L> <mode> <queries.f32> <nq> <out.u32>
//       ComputeService::search of each query (one call per query) and
//       search_batch of all of them; writes nq*k ids (0xFFFFFFFF padded) from
//       search, then the same from search_batch
//   service_check insert <prefix> <dim> <k> <L> <vectors.f32> <n> <first_id> <store_prefix>
//       ComputeService::insert of n vectors (ids first_id ...), then store_index
//       to store_prefix; prints "inserted <count> vectors_inserted <status>"
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <string>
#include <vector>

#include "dvs_b200_service.hpp"

namespace {

std::vector<float> read_f32(const std::string& path, size_t count) {
  std::vector<float> v(count);
  std::ifstream f(path, std::ios::binary);
  f.read(reinterpret_cast<char*>(v.data()), std::streamsize(count * sizeof(float)));
  if (!f) throw std::runtime_error("short read of " + path);
  return v;
}

dvs::Configuration base(uint32_t dim, uint32_t k, uint32_t L, const std::string& mode) {
  dvs::Configuration c;
  c.dim = dim;
  c.k = k;
  c.beam_width = L;
  c.search_mode = mode;
  c.rabitq_bits = 4;
  return c;
}

template <class F>
void expect_config_error(const char* name, F f) {
  try {
    f();
    std::cout << name << ": no error\n";
  } catch (const dvs::ConfigError& e) {
    std::cout << name << ": " << e.what() << "\n";
  }
}

int config_checks() {
  expect_config_error("required", [] {
    dvs::Configuration c;
    c.validate();
  });
  expect_config_error("mode", [] {
    dvs::Configuration c = base(8, 10, 64, "cpu");
    c.validate();
  });
  expect_config_error("bits", [] {
    dvs::Configuration c = base(8, 10, 64, "rabitq_gpu");
    c.rabitq_bits = 3;
    c.validate();
  });
  expect_config_error("load_store", [] {
    dvs::Configuration c = base(8, 10, 64, "exact_gpu");
    c.load_index = c.store_index = true;
    c.index_prefix = "x";
    c.validate();
  });
  expect_config_error("prefix", [] {
    dvs::Configuration c = base(8, 10, 64, "exact_gpu");
    c.load_index = true;
    c.validate();
  });
  expect_config_error("beam", [] {
    dvs::Configuration c = base(8, 10, 5, "exact_gpu");
    c.validate();
  });
  {
    dvs::Configuration c = base(8, 10, 64, "RABITQ_GPU");
    c.validate();
    std::cout << "normalized: " << c.search_mode << "\n";
    c.data_path = "/data/sift/base.fvecs";
    c.R = 32;
    c.beam_width_construction = 128;
    std::cout << "prefix: " << c.resolved_index_prefix() << "\n";
  }
  {
    dvs::ComputeService svc(base(8, 10, 64, "exact_gpu"));
    std::string msg;
    const bool ok = svc.load_index("/nonexistent/index_prefix", &msg);
    std::cout << "load_missing: " << (ok ? "ok" : "failed") << " (" << (msg.empty() ? "no message" : "message")
              << ")\n";
    try {
      svc.search(std::vector<float>(7, 0.f), 5);
      std::cout << "dim: no error\n";
    } catch (const std::invalid_argument& e) {
      std::cout << "dim: " << e.what() << "\n";
    }
    try {
      svc.insert({{1u, std::vector<float>(9, 0.f)}});
      std::cout << "insert_dim: no error\n";
    } catch (const std::invalid_argument& e) {
      std::cout << "insert_dim: " << e.what() << "\n";
    }
    try {
      svc.search(std::vector<float>(8, 0.f), 5);
      std::cout << "no_index: no error\n";
    } catch (const dvs::Error& e) {
      std::cout << "no_index: " << e.what() << "\n";
    }
    const auto st = svc.status();
    std::cout << "status: " << st.state << " " << st.vectors_inserted << " " << st.dimension << "\n";
  }
  return 0;
}

int search(char** a) {
  const std::string prefix = a[2], mode = a[6];
  const uint32_t dim = uint32_t(std::atoi(a[3])), k = uint32_t(std::atoi(a[4])), L = uint32_t(std::atoi(a[5]));
  const size_t nq = size_t(std::atoll(a[8]));
  dvs::Configuration c = base(dim, k, L, mode);
  c.index_prefix = prefix;
  c.load_index = true;
  dvs::ComputeService svc(c);
  const std::vector<float> q = read_f32(a[7], nq * dim);
  std::vector<uint32_t> out(2 * nq * k, 0xFFFFFFFFu);
  for (size_t i = 0; i < nq; ++i) {
    const std::vector<uint32_t> r = svc.search(std::vector<float>(q.begin() + i * dim, q.begin() + (i + 1) * dim), k);
    for (size_t j = 0; j < r.size(); ++j) out[i * k + j] = r[j];
  }
  const auto rb = svc.search_batch(q.data(), nq, k);
  for (size_t i = 0; i < nq; ++i)
    for (size_t j = 0; j < rb[i].size(); ++j) out[(nq + i) * k + j] = rb[i][j];
  std::ofstream f(a[9], std::ios::binary);
  f.write(reinterpret_cast<const char*>(out.data()), std::streamsize(out.size() * 4));
  const auto st = svc.statistics();
  std::cout << "queries " << st.processed_queries << " expansions " << st.visited_neighborlists << "\n";
  return 0;
}

int insert(char** a) {
  const std::string prefix = a[2];
  const uint32_t dim = uint32_t(std::atoi(a[3])), k = uint32_t(std::atoi(a[4])), L = uint32_t(std::atoi(a[5]));
  const size_t n = size_t(std::atoll(a[7]));
  const uint32_t first = uint32_t(std::atoll(a[8]));
  dvs::Configuration c = base(dim, k, L, "rabitq_gpu");
  c.index_prefix = prefix;
  c.load_index = true;
  c.beam_width_construction = 64;
  dvs::ComputeService svc(c);
  const std::vector<float> x = read_f32(a[6], n * dim);
  std::vector<dvs::ComputeService::InsertItem> batch;
  for (size_t i = 0; i < n; ++i)
    batch.push_back({first + uint32_t(i), std::vector<float>(x.begin() + i * dim, x.begin() + (i + 1) * dim)});
  const size_t got = svc.insert(batch);
  std::string msg;
  const bool ok = svc.store_index(a[9], &msg);
  std::cout << "inserted " << got << " vectors_inserted " << svc.status().vectors_inserted << " store "
            << (ok ? "ok" : msg) << "\n";
  return ok ? 0 : 1;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    const std::string cmd = argc > 1 ? argv[1] : "";
    if (cmd == "config") return config_checks();
    if (cmd == "search" && argc == 10) return search(argv);
    if (cmd == "insert" && argc == 10) return insert(argv);
    std::cerr << "usage: service_check config | search ... | insert ...\n";
    return 2;
  } catch (const std::exception& e) {
    std::cerr << "error: " << e.what() << "\n";
    return 1;
  }
}
