// Timed CPU baseline.  TEST / MEASUREMENT INFRASTRUCTURE ONLY (bench.py's
// cpu_baseline leg and `--impl reference` arm).
//
// The reference's only CPU Vamana search is the offline builder's beam_search
// (tools/vamana_offline_builder.cc:523-625): exact L2 with the AVX l2_squared
// (:313-345), std::unordered_set visited/expanded sets, a std::sort of the beam
// after every expansion, and the whole visited set sorted at the end; its first
// k entries are the answer (the builder's recall test, :1387-1440).  The
// reference cannot be compiled here (Eigen, Boost and oneTBB share its
// translation unit), so this file restates that function line for line and runs
// one query per task over the host threads with the reference's atomic-counter
// parallel_for (:198-227).  It is compiled -O3 -mavx2 -mfma like the reference's
// -march=native AVX2 build, without -ffast-math.  Neighbour lists are read
// without the per-node mutex: the graph does not change during a query run.

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <thread>
#include <unordered_set>
#include <vector>

namespace {

constexpr uint32_t kEmpty = 0xFFFFFFFFu;

float l2_squared_avx(const float* a, const float* b, uint32_t dim) {
  __m256 sum = _mm256_setzero_ps();
  uint32_t i = 0;
  for (; i + 16 <= dim; i += 16) {
    __m256 v1 = _mm256_loadu_ps(a + i);
    __m256 v2 = _mm256_loadu_ps(b + i);
    __m256 d = _mm256_sub_ps(v1, v2);
    sum = _mm256_add_ps(sum, _mm256_mul_ps(d, d));
    v1 = _mm256_loadu_ps(a + i + 8);
    v2 = _mm256_loadu_ps(b + i + 8);
    d = _mm256_sub_ps(v1, v2);
    sum = _mm256_add_ps(sum, _mm256_mul_ps(d, d));
  }
  alignas(32) float tmp[8];
  _mm256_store_ps(tmp, sum);
  float result = tmp[0] + tmp[1] + tmp[2] + tmp[3] + tmp[4] + tmp[5] + tmp[6] + tmp[7];
  for (; i < dim; ++i) {
    const float d = a[i] - b[i];
    result += d * d;
  }
  return result;
}

using Pair = std::pair<float, uint32_t>;

// beam_search of the builder; returns the number of visited nodes and writes the
// first k ids of the sorted visited set.
uint32_t beam_search(const float* X, uint32_t dim, const uint32_t* adj, uint32_t R, uint32_t medoid,
                     const float* query, uint32_t L, uint32_t k, uint32_t* out_ids) {
  std::vector<Pair> all_visited, beam;
  std::unordered_set<uint32_t> visited, expanded;
  const float md = l2_squared_avx(query, X + size_t(medoid) * dim, dim);
  beam.push_back({md, medoid});
  all_visited.push_back({md, medoid});
  visited.insert(medoid);
  std::vector<uint32_t> nbrs, unvisited;
  for (;;) {
    ptrdiff_t best_pos = -1;
    for (size_t i = 0; i < beam.size(); ++i) {
      if (expanded.count(beam[i].second) == 0) {
        best_pos = ptrdiff_t(i);
        break;
      }
    }
    if (best_pos < 0) break;
    const uint32_t best = beam[best_pos].second;
    expanded.insert(best);
    nbrs.clear();
    const uint32_t* row = adj + size_t(best) * R;
    for (uint32_t j = 0; j < R; ++j)
      if (row[j] != kEmpty) nbrs.push_back(row[j]);
    unvisited.clear();
    for (uint32_t nb : nbrs) {
      if (visited.count(nb)) continue;
      visited.insert(nb);
      unvisited.push_back(nb);
    }
    for (uint32_t nb : unvisited) {
      const float d = l2_squared_avx(query, X + size_t(nb) * dim, dim);
      beam.push_back({d, nb});
      all_visited.push_back({d, nb});
    }
    std::sort(beam.begin(), beam.end());
    if (beam.size() > L) beam.resize(L);
  }
  std::sort(all_visited.begin(), all_visited.end());
  for (uint32_t i = 0; i < k; ++i) out_ids[i] = i < all_visited.size() ? all_visited[i].second : kEmpty;
  return uint32_t(all_visited.size());
}

}  // namespace

extern "C" int orc_cpu_beam_search_batch(const float* X, uint64_t n, uint32_t dim, const uint32_t* adj, uint32_t R,
                                         uint32_t medoid, const float* queries, uint32_t nq, uint32_t L, uint32_t k,
                                         int threads, uint32_t* out_ids, uint32_t* out_visited) {
  (void)n;
  size_t nt = threads > 0 ? size_t(threads) : std::max<size_t>(1, std::thread::hardware_concurrency());
  nt = std::min<size_t>(nt, std::max<uint32_t>(nq, 1));
  std::atomic<size_t> next{0};
  auto work = [&]() {
    for (;;) {
      const size_t q = next.fetch_add(1);
      if (q >= nq) return;
      const uint32_t v = beam_search(X, dim, adj, R, medoid, queries + q * dim, L, k, out_ids + q * k);
      if (out_visited) out_visited[q] = v;
    }
  };
  std::vector<std::thread> pool;
  for (size_t t = 1; t < nt; ++t) pool.emplace_back(work);
  work();
  for (auto& th : pool) th.join();
  return 0;
}
