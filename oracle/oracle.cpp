// CPU oracle for the DVSTOR `rabitq_gpu` query path and the offline builder that
// produces its index.
//
// TEST INFRASTRUCTURE ONLY.  tests/, __graft_entry__.smoke() and bench.py's
// cpu_baseline / `--impl reference` leg load this library as the checker or as
// the timed CPU baseline.  The product (dvstor_b200/) never links, loads or calls
// it.
//
// Every function restates one piece of the reference (paths are relative to the
// reference project root) with its floating-point order written out, so that the
// CUDA path can reproduce it bit for bit:
//   * fmaf() wherever the reference's nvcc build contracts `acc += a * b`
//     (nvcc defaults to --fmad=true and the reference passes no flag against it);
//   * 4-lane cooperative-groups tiles reduce with cg::reduce's xor butterfly
//     (mask 2, then mask 1), so a tile sum is (s0 + s2) + (s1 + s3);
//   * host-side code that the reference writes as separate multiply and add is
//     kept separate (this file is compiled with -ffp-contract=off).
// The reference ships no golden vectors; tests/golden/ holds outputs of the
// reference's own GPU kernels (compiled from its sources into oracle/_ref) on
// seeded inputs, and the CPU tests check this file against them.

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <limits>
#include <mutex>
#include <numeric>
#include <queue>
#include <random>
#include <string>
#include <thread>
#include <unordered_set>
#include <vector>

namespace {

constexpr uint32_t kEmpty = 0xFFFFFFFFu;         // empty adjacency slot
constexpr uint32_t kRabitqSearchBeamSlack = 64;  // src/vamana/vamana.hh:33

// ----------------------------------------------------------------------------
// Threading helper: the reference's parallel_for (tools/vamana_offline_builder.cc
// :198-227) hands out indices from one atomic counter.
// ----------------------------------------------------------------------------
template <class Fn>
void parallel_for(size_t begin, size_t end, int threads, Fn&& fn) {
  size_t nt = threads > 0 ? size_t(threads) : std::max<size_t>(1, std::thread::hardware_concurrency());
  if (nt <= 1 || end <= begin + 1) {
    for (size_t i = begin; i < end; ++i) fn(i);
    return;
  }
  nt = std::min(nt, end - begin);
  std::atomic<size_t> next{begin};
  std::vector<std::thread> pool;
  pool.reserve(nt);
  for (size_t t = 0; t < nt; ++t) {
    pool.emplace_back([&]() {
      for (;;) {
        const size_t i = next.fetch_add(1);
        if (i >= end) return;
        fn(i);
      }
    });
  }
  for (auto& th : pool) th.join();
}

inline float tile4(const float s[4]) { return (s[0] + s[2]) + (s[1] + s[3]); }

// ----------------------------------------------------------------------------
// Distances
// ----------------------------------------------------------------------------

// Exact squared L2 in the order of batch_l2_squared_distance_kernel<4>
// (src/gpu/kernels/distance_kernels.cuh:38-81): lane t of a 4-lane tile walks the
// float4 chunks i = t, t+4, ... and accumulates the four components in order,
// then the tail dims base+t; the tile is reduced with the xor butterfly.
float l2_ref(const float* q, const float* x, uint32_t dim) {
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t n4 = dim / 4;
  for (uint32_t i = 0; i < n4; ++i) {
    float& acc = s[i & 3];
    for (uint32_t k = 0; k < 4; ++k) {
      const float d = q[4 * i + k] - x[4 * i + k];
      acc = std::fmaf(d, d, acc);
    }
  }
  for (uint32_t i = n4 * 4; i < dim; ++i) {
    const float d = q[i] - x[i];
    float& acc = s[(i - n4 * 4) & 3];
    acc = std::fmaf(d, d, acc);
  }
  return tile4(s);
}

// Medoid seed distance of Vamana::knn (src/vamana/vamana.hh:118), computed on the
// host by L2Distance::dist (src/common/distance.hh:80-113, 151-153): eight AVX
// lanes over 16-float chunks (first half, then second half), a left-to-right
// horizontal sum, then the scalar tail.  The reference builds this with
// -march=native -ffast-math, which lets GCC contract the multiply-add; this
// restatement contracts (fmaf) and keeps the written summation order.
float seed_l2(const float* a, const float* b, uint32_t dim) {
  const uint32_t q16 = dim >> 4 << 4;
  float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (uint32_t c = 0; c < q16; c += 16) {
    for (int l = 0; l < 8; ++l) {
      const float d = a[c + l] - b[c + l];
      lane[l] = std::fmaf(d, d, lane[l]);
    }
    for (int l = 0; l < 8; ++l) {
      const float d = a[c + 8 + l] - b[c + 8 + l];
      lane[l] = std::fmaf(d, d, lane[l]);
    }
  }
  float r = lane[0];
  for (int l = 1; l < 8; ++l) r = r + lane[l];
  for (uint32_t i = q16; i < dim; ++i) {
    const float d = a[i] - b[i];
    r = std::fmaf(d, d, r);
  }
  return r;
}

// IPDistance::dist (src/common/distance.hh:120-151, 155-159): 1 - dot with the
// same eight-lane layout and a separately accumulated tail.
float seed_ip(const float* a, const float* b, uint32_t dim) {
  const uint32_t q16 = dim >> 4 << 4;
  float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (uint32_t c = 0; c < q16; c += 16) {
    for (int l = 0; l < 8; ++l) lane[l] = std::fmaf(a[c + l], b[c + l], lane[l]);
    for (int l = 0; l < 8; ++l) lane[l] = std::fmaf(a[c + 8 + l], b[c + 8 + l], lane[l]);
  }
  float res = lane[0];
  for (int l = 1; l < 8; ++l) res = res + lane[l];
  float tail = 0.f;
  for (uint32_t i = q16; i < dim; ++i) tail = std::fmaf(a[i], b[i], tail);
  return 1.0f - (res + tail);
}

// ----------------------------------------------------------------------------
// RaBitQ query side
// ----------------------------------------------------------------------------

// q' = P^T q with P column-major (src/gpu/gpu_kernel_launcher.cu:289-297 calls
// cublasSgemv(OP_T, D, D, P, ld=D)).  cuBLAS's summation order is not public;
// this restatement fixes one order (a sequential fmaf chain over i) that the
// CUDA path reproduces exactly, and the tests hold it to a tolerance against
// the reference's cuBLAS result.
void rotate(const float* P, const float* x, uint32_t dim, float* out) {
  for (uint32_t j = 0; j < dim; ++j) {
    const float* col = P + size_t(j) * dim;
    float acc = 0.f;
    for (uint32_t i = 0; i < dim; ++i) acc = std::fmaf(col[i], x[i], acc);
    out[j] = acc;
  }
}

// rabitq_query_prepare_kernel<4,B> (src/gpu/kernels/distance_kernels.cuh:470-501).
void query_factors(const float* qr, const float* c, uint32_t dim, uint32_t bits, float* f3) {
  float sq[4] = {0, 0, 0, 0}, sm[4] = {0, 0, 0, 0};
  for (uint32_t j = 0; j < dim; ++j) {
    const float diff = qr[j] - c[j];
    sq[j & 3] = std::fmaf(diff, diff, sq[j & 3]);
    sm[j & 3] = sm[j & 3] + qr[j];
  }
  const float sqr_norm = tile4(sq);
  const float sumq = tile4(sm);
  const float c_b = -static_cast<float>((1u << bits) - 1u) / 2.0f;
  const float c_1 = -static_cast<float>((1u << 1) - 1u) / 2.0f;
  f3[0] = sqr_norm;
  f3[1] = c_1 * sumq;
  f3[2] = c_b * sumq;
}

// batch_rabitq_distance_kernel<4,B> (src/gpu/kernels/distance_kernels.cuh:95-137):
// lane t of the tile sums dims j = t, t+4, ...; the tile is reduced with the
// butterfly; the estimate is add_o + q.add + rescale_o * (dot + k1xSumq*(2^B-1)),
// which nvcc contracts to fma(rescale_o, fma(k1xSumq, 2^B-1, dot), add_o + q.add).
// batch_rabitq_8bit_distance_kernel<4> (src/gpu/kernels/distance_kernels.cuh:181-221):
// one char4 chunk (4 dims) per step, lane t takes chunks i = t, t+4, ...; only
// the first 4*floor(dim/4) dims take part.  Per chunk the sum
// x0*q0 + x1*q1 + x2*q2 + x3*q3 is contracted by nvcc (left to right) to
// fma(x3,q3, fma(x2,q2, fma(x0,q0, x1*q1))) and added to the lane's sum.
float rabitq_estimate_8bit(const float* qr, const float* f3, const uint8_t* rec, uint32_t dim) {
  float add_o, rescale_o;
  std::memcpy(&add_o, rec + dim, 4);
  std::memcpy(&rescale_o, rec + dim + 4, 4);
  float s[4] = {0, 0, 0, 0};
  for (uint32_t i = 0; i < dim / 4; ++i) {
    const uint8_t* d = rec + 4 * i;
    const float* q = qr + 4 * i;
    float t = static_cast<float>(d[1]) * q[1];
    t = std::fmaf(static_cast<float>(d[0]), q[0], t);
    t = std::fmaf(static_cast<float>(d[2]), q[2], t);
    t = std::fmaf(static_cast<float>(d[3]), q[3], t);
    s[i & 3] = s[i & 3] + t;
  }
  const float dot = tile4(s);
  return std::fmaf(rescale_o, std::fmaf(f3[1], 255.0f, dot), add_o + f3[0]);
}

float rabitq_estimate_one(const float* qr, const float* f3, const uint8_t* rec, uint32_t dim, uint32_t bits) {
  if (bits == 8) return rabitq_estimate_8bit(qr, f3, rec, dim);
  const uint32_t packed = (bits * dim + 7) / 8;
  float add_o, rescale_o;
  std::memcpy(&add_o, rec + packed, 4);
  std::memcpy(&rescale_o, rec + packed + 4, 4);
  const uint32_t mask = (1u << bits) - 1u;
  float s[4] = {0, 0, 0, 0};
  for (uint32_t j = 0; j < dim; ++j) {
    const uint32_t bit_idx = j * bits;
    const uint32_t byte_idx = bit_idx / 8;
    const uint32_t bit_off = bit_idx % 8;
    uint32_t chunk = rec[byte_idx];
    if (bit_off + bits > 8 && byte_idx + 1 < packed) chunk |= uint32_t(rec[byte_idx + 1]) << 8;
    const float val = static_cast<float>((chunk >> bit_off) & mask);
    s[j & 3] = std::fmaf(val, qr[j], s[j & 3]);
  }
  const float dot = tile4(s);
  const float k1 = static_cast<float>((1u << bits) - 1u);
  return std::fmaf(rescale_o, std::fmaf(f3[1], k1, dot), add_o + f3[0]);
}

// ----------------------------------------------------------------------------
// RaBitQ build side (tools/vamana_offline_builder.cc:864-1102)
// ----------------------------------------------------------------------------

constexpr float kTightStart[9] = {0.0f, 0.15f, 0.20f, 0.52f, 0.59f, 0.71f, 0.75f, 0.77f, 0.81f};

// best_rescale_factor (tools/vamana_offline_builder.cc:889-947).
double best_rescale_factor(const float* abs_unit, size_t dim, size_t bits) {
  constexpr double kEps = 1e-5;
  constexpr int kNEnum = 10;
  const double max_o = *std::max_element(abs_unit, abs_unit + dim);
  if (max_o <= 0.0) return 0.0;
  const double t_end = static_cast<double>(((1u << bits) - 1u) + kNEnum) / max_o;
  const double t_start = t_end * kTightStart[bits];
  std::vector<int> cur_o_bar(dim);
  double sqr_denominator = static_cast<double>(dim) * 0.25;
  double numerator = 0.0;
  for (size_t i = 0; i < dim; ++i) {
    const int cur = static_cast<int>((t_start * abs_unit[i]) + kEps);
    cur_o_bar[i] = cur;
    sqr_denominator += static_cast<double>(cur) * cur + cur;
    numerator += (static_cast<double>(cur) + 0.5) * abs_unit[i];
  }
  std::priority_queue<std::pair<double, size_t>, std::vector<std::pair<double, size_t>>, std::greater<>> next_t;
  for (size_t i = 0; i < dim; ++i)
    if (abs_unit[i] > 0.0f) next_t.emplace(static_cast<double>(cur_o_bar[i] + 1) / abs_unit[i], i);
  double max_ip = 0.0, best_t = 0.0;
  while (!next_t.empty()) {
    const auto [cur_t, update_id] = next_t.top();
    next_t.pop();
    cur_o_bar[update_id]++;
    const int update_o_bar = cur_o_bar[update_id];
    sqr_denominator += 2.0 * update_o_bar;
    numerator += abs_unit[update_id];
    const double cur_ip = numerator / std::sqrt(sqr_denominator);
    if (cur_ip > max_ip) {
      max_ip = cur_ip;
      best_t = cur_t;
    }
    if (update_o_bar < static_cast<int>((1u << bits) - 1u)) {
      const double t_next = static_cast<double>(update_o_bar + 1) / abs_unit[update_id];
      if (t_next < t_end) next_t.emplace(t_next, update_id);
    }
  }
  return best_t;
}

// get_const_scaling_factors (tools/vamana_offline_builder.cc:949-973).
double t_const(size_t dim, size_t bits, uint64_t seed) {
  constexpr size_t n_samples = 1000;
  std::mt19937_64 rng(seed);
  std::normal_distribution<float> normal(0.0f, 1.0f);
  std::vector<float> sample(dim), abs_unit(dim);
  double total = 0.0;
  for (size_t s = 0; s < n_samples; ++s) {
    double norm_sqr = 0.0;
    for (size_t d = 0; d < dim; ++d) {
      sample[d] = normal(rng);
      norm_sqr += static_cast<double>(sample[d]) * sample[d];
    }
    const double norm = std::sqrt(norm_sqr);
    const double inv_norm = norm > 0.0 ? (1.0 / norm) : 0.0;
    for (size_t d = 0; d < dim; ++d) abs_unit[d] = std::fabs(static_cast<float>(sample[d] * inv_norm));
    total += best_rescale_factor(abs_unit.data(), dim, bits);
  }
  return total / static_cast<double>(n_samples);
}

// Random matrix of init_rabitq (tools/vamana_offline_builder.cc:991-996):
// random_mat(i, j) = normal(rng) with i outer, stored column-major.
void gaussian_matrix(uint32_t dim, int seed, double* out_colmajor) {
  std::mt19937 rng(seed);
  std::normal_distribution<float> normal(0.0f, 1.0f);
  for (uint32_t i = 0; i < dim; ++i)
    for (uint32_t j = 0; j < dim; ++j) out_colmajor[i + size_t(j) * dim] = normal(rng);
}

// P of init_rabitq (tools/vamana_offline_builder.cc:998-1005): Q of a Householder
// QR of the Gaussian matrix, each column negated where R(i,i) < 0.  Eigen is not
// available here; this is an independent double-precision Householder QR.  The
// positive-diagonal QR factor is unique, so P agrees with Eigen's to rounding.
void rotation_matrix(uint32_t dim, int seed, float* P_out) {
  const size_t D = dim;
  std::vector<double> A(D * D), A0(D * D), Q(D * D, 0.0), v(D);
  gaussian_matrix(dim, seed, A.data());
  A0 = A;
  std::vector<std::vector<double>> vs(D);
  for (size_t k = 0; k < D; ++k) {
    double nrm = 0.0;
    for (size_t i = k; i < D; ++i) nrm += A[i + k * D] * A[i + k * D];
    nrm = std::sqrt(nrm);
    const double x0 = A[k + k * D];
    const double alpha = x0 >= 0 ? -nrm : nrm;
    std::vector<double> vk(D - k);
    for (size_t i = k; i < D; ++i) vk[i - k] = A[i + k * D];
    vk[0] -= alpha;
    double vn = 0.0;
    for (double t : vk) vn += t * t;
    vn = std::sqrt(vn);
    if (vn > 0) {
      for (double& t : vk) t /= vn;
      for (size_t c = k; c < D; ++c) {
        double dot = 0.0;
        for (size_t i = k; i < D; ++i) dot += vk[i - k] * A[i + c * D];
        for (size_t i = k; i < D; ++i) A[i + c * D] -= 2.0 * vk[i - k] * dot;
      }
    }
    vs[k] = std::move(vk);
  }
  for (size_t i = 0; i < D; ++i) Q[i + i * D] = 1.0;
  for (size_t kk = D; kk-- > 0;) {
    const auto& vk = vs[kk];
    for (size_t c = 0; c < D; ++c) {
      double dot = 0.0;
      for (size_t i = kk; i < D; ++i) dot += vk[i - kk] * Q[i + c * D];
      for (size_t i = kk; i < D; ++i) Q[i + c * D] -= 2.0 * vk[i - kk] * dot;
    }
  }
  for (size_t c = 0; c < D; ++c) {
    double r = 0.0;  // R(c, c) = Q(:, c)^T A0(:, c)
    for (size_t i = 0; i < D; ++i) r += Q[i + c * D] * A0[i + c * D];
    const double sgn = r < 0.0 ? -1.0 : 1.0;
    for (size_t i = 0; i < D; ++i) P_out[i + c * D] = static_cast<float>(sgn * Q[i + c * D]);
  }
}

// Centroid of init_rabitq (tools/vamana_offline_builder.cc:1008-1013): a float
// sum over the vectors in order, divided by n.
void centroid(const float* X, size_t n, uint32_t dim, float* out) {
  std::fill(out, out + dim, 0.0f);
  for (size_t i = 0; i < n; ++i)
    for (uint32_t d = 0; d < dim; ++d) out[d] = out[d] + X[i * dim + d];
  for (uint32_t d = 0; d < dim; ++d) out[d] = out[d] / static_cast<float>(n);
}

// rabitq_quantize_vector (tools/vamana_offline_builder.cc:1030-1102) given the
// rotated vector.  Record layout: [packed (B*D+7)/8 | f32 add | f32 rescale].
void quantize_rotated(const float* rotated, const float* c_rot, double tc, uint32_t dim, uint32_t bits,
                      uint8_t* out) {
  constexpr double kEps = 1e-5;
  const uint32_t packed = (bits * dim + 7) / 8;
  std::vector<float> delta(dim);
  for (uint32_t i = 0; i < dim; ++i) delta[i] = rotated[i] - c_rot[i];
  float l2_sqr = 0.0f;
  for (uint32_t i = 0; i < dim; ++i) l2_sqr = l2_sqr + delta[i] * delta[i];
  const float l2_norm = std::sqrt(l2_sqr);
  std::vector<uint8_t> qv(dim, 0);
  float ip_norm = 0.0f;
  const uint32_t cap = (1u << (bits - 1)) - 1u;
  for (uint32_t i = 0; i < dim; ++i) {
    const float abs_o = l2_norm > 0.0f ? std::fabs(delta[i] / l2_norm) : 0.0f;
    int val = static_cast<int>((tc * abs_o) + kEps);
    if (val >= static_cast<int>(1u << (bits - 1))) val = static_cast<int>(cap);
    qv[i] = static_cast<uint8_t>(val);
    ip_norm = ip_norm + (static_cast<float>(val) + 0.5f) * abs_o;
  }
  const float ip_norm_inv = ip_norm == 0.0f ? 1.0f : (1.0f / ip_norm);
  for (uint32_t i = 0; i < dim; ++i) {
    if (delta[i] >= 0.0f)
      qv[i] = static_cast<uint8_t>(qv[i] + (1u << (bits - 1)));
    else
      qv[i] = static_cast<uint8_t>((~qv[i]) & cap);
  }
  std::memset(out, 0, packed);
  for (uint32_t i = 0; i < dim; ++i) {
    const uint32_t bit_idx = i * bits, byte_idx = bit_idx / 8, bit_off = bit_idx % 8;
    out[byte_idx] |= static_cast<uint8_t>(qv[i] << bit_off);
    if (bit_off + bits > 8 && byte_idx + 1 < packed) out[byte_idx + 1] |= static_cast<uint8_t>(qv[i] >> (8 - bit_off));
  }
  const float cb = -(static_cast<float>(1u << (bits - 1)) - 0.5f);
  float ip_resi = 0.0f, ip_cent = 0.0f;
  for (uint32_t i = 0; i < dim; ++i) {
    const float xu_cb = static_cast<float>(qv[i]) + cb;
    ip_resi = ip_resi + delta[i] * xu_cb;
    ip_cent = ip_cent + c_rot[i] * xu_cb;
  }
  if (ip_resi == 0.0f) ip_resi = std::numeric_limits<float>::infinity();
  const float add_f = l2_sqr + 2.0f * l2_sqr * ip_cent / ip_resi;
  const float rescale_f = ip_norm_inv * -2.0f * l2_norm;
  std::memcpy(out + packed, &add_f, 4);
  std::memcpy(out + packed + 4, &rescale_f, 4);
}

// ----------------------------------------------------------------------------
// Vamana graph builder (tools/vamana_offline_builder.cc:473-861)
// ----------------------------------------------------------------------------

using Pair = std::pair<float, uint32_t>;

// compute_medoid (tools/vamana_offline_builder.cc:473-507).
size_t compute_medoid(const float* X, size_t n, uint32_t dim) {
  const size_t sample_size = std::min<size_t>(n, 10000);
  std::vector<size_t> idx(n);
  std::iota(idx.begin(), idx.end(), 0);
  if (sample_size < n) {
    std::mt19937 rng(42);
    std::shuffle(idx.begin(), idx.end(), rng);
    idx.resize(sample_size);
  }
  std::vector<float> c(dim, 0.0f);
  for (size_t i : idx)
    for (uint32_t d = 0; d < dim; ++d) c[d] = c[d] + X[i * dim + d];
  for (uint32_t d = 0; d < dim; ++d) c[d] = c[d] / static_cast<float>(sample_size);
  size_t best = 0;
  float best_dist = std::numeric_limits<float>::max();
  for (size_t i = 0; i < n; ++i) {
    const float d = l2_ref(X + i * dim, c.data(), dim);
    if (d < best_dist) {
      best_dist = d;
      best = i;
    }
  }
  return best;
}

// Random R-regular init (tools/vamana_offline_builder.cc:700-718); the degree is
// capped at n-1 so that a tiny dataset cannot spin forever.
void random_init(size_t n, uint32_t R, size_t seed, std::vector<std::vector<uint32_t>>& g) {
  g.assign(n, {});
  const size_t deg = std::min<size_t>(R, n > 0 ? n - 1 : 0);
  std::mt19937 init_rng(seed + 1);
  std::uniform_int_distribution<size_t> dist(0, n - 1);
  for (size_t i = 0; i < n; ++i) {
    g[i].reserve(R);
    while (g[i].size() < deg) {
      const size_t j = dist(init_rng);
      if (j == i) continue;
      bool dup = false;
      for (uint32_t k : g[i])
        if (k == static_cast<uint32_t>(j)) {
          dup = true;
          break;
        }
      if (!dup) g[i].push_back(static_cast<uint32_t>(j));
    }
  }
}

// beam_search (tools/vamana_offline_builder.cc:523-625): returns every node
// whose distance was computed, sorted by (distance, id).
std::vector<Pair> build_beam_search(const std::vector<std::vector<uint32_t>>& g, const float* X, uint32_t dim,
                                    size_t medoid, const float* q, uint32_t L) {
  std::vector<Pair> all_visited, beam;
  std::unordered_set<uint32_t> visited, expanded;
  const float md = l2_ref(q, X + medoid * dim, dim);
  beam.push_back({md, uint32_t(medoid)});
  all_visited.push_back({md, uint32_t(medoid)});
  visited.insert(uint32_t(medoid));
  for (;;) {
    ptrdiff_t best = -1;
    for (size_t i = 0; i < beam.size(); ++i)
      if (!expanded.count(beam[i].second)) {
        best = ptrdiff_t(i);
        break;
      }
    if (best < 0) break;
    const uint32_t u = beam[best].second;
    expanded.insert(u);
    for (uint32_t nb : g[u]) {
      if (visited.count(nb)) continue;
      visited.insert(nb);
      const float d = l2_ref(q, X + size_t(nb) * dim, dim);
      beam.push_back({d, nb});
      all_visited.push_back({d, nb});
    }
    std::sort(beam.begin(), beam.end());
    if (beam.size() > L) beam.resize(L);
  }
  std::sort(all_visited.begin(), all_visited.end());
  return all_visited;
}

// robust_prune (tools/vamana_offline_builder.cc:634-663).
std::vector<uint32_t> robust_prune(const float* X, uint32_t dim, uint32_t source, const std::vector<Pair>& cand,
                                   float alpha, uint32_t R) {
  std::vector<uint32_t> sel;
  sel.reserve(R);
  for (const auto& [cd, cid] : cand) {
    if (cid == source) continue;
    if (sel.size() >= R) break;
    bool pruned = false;
    for (uint32_t s : sel) {
      const float d = l2_ref(X + size_t(s) * dim, X + size_t(cid) * dim, dim);
      if (alpha * d <= cd) {
        pruned = true;
        break;
      }
    }
    if (!pruned) sel.push_back(cid);
  }
  return sel;
}

// Batch sizes of the deterministic batched build: 1, 2, 4, ... doubling up to
// `cap`.  Within a batch every node searches the graph as it stood when the
// batch began; the reference's parallel_for lets ~threads inserts race on a
// graph that changes under them, so its result is not reproducible at all.
std::vector<std::pair<size_t, size_t>> batch_schedule(size_t n, size_t cap) {
  std::vector<std::pair<size_t, size_t>> out;
  size_t pos = 0, sz = 1;
  cap = std::max<size_t>(cap, 1);
  while (pos < n) {
    const size_t b = std::min(std::min(sz, cap), n - pos);
    out.push_back({pos, pos + b});
    pos += b;
    sz = std::min(sz * 2, cap);
  }
  return out;
}

// build_vamana_graph (tools/vamana_offline_builder.cc:673-861) in batched form:
//   (a) every node of the batch runs beam_search on the graph frozen at batch start;
//   (b) candidates = visited set + the node's current neighbours (distances
//       recomputed), sorted by (distance, id), adjacent duplicates removed,
//       RobustPrune with build alpha 1.0 (tools/vamana_offline_builder.cc:723);
//   (c) the pruned lists replace the batch nodes' lists;
//   (d) reverse edges are grouped by target in batch order; a target that would
//       exceed R keeps RobustPrune(own list + additions), otherwise appends.
void build_graph(const float* X, size_t n, uint32_t dim, uint32_t R, uint32_t L, float alpha, size_t seed,
                 size_t batch_cap, int threads, std::vector<std::vector<uint32_t>>& g, size_t& medoid) {
  medoid = compute_medoid(X, n, dim);
  std::vector<size_t> order(n);
  std::iota(order.begin(), order.end(), 0);
  {
    std::mt19937 rng(seed);
    std::shuffle(order.begin(), order.end(), rng);
  }
  random_init(n, R, seed, g);
  for (auto [b0, b1] : batch_schedule(n, batch_cap)) {
    const size_t nb = b1 - b0;
    std::vector<std::vector<uint32_t>> fresh(nb);
    parallel_for(0, nb, threads, [&](size_t t) {
      const size_t u = order[b0 + t];
      const float* q = X + u * dim;
      auto cand = build_beam_search(g, X, dim, medoid, q, L);
      for (uint32_t e : g[u]) cand.push_back({l2_ref(q, X + size_t(e) * dim, dim), e});
      std::sort(cand.begin(), cand.end());
      cand.erase(std::unique(cand.begin(), cand.end(),
                             [](const Pair& a, const Pair& b) { return a.second == b.second; }),
                 cand.end());
      fresh[t] = robust_prune(X, dim, uint32_t(u), cand, alpha, R);
    });
    for (size_t t = 0; t < nb; ++t) g[order[b0 + t]] = fresh[t];
    // reverse edges grouped by target, in batch order
    std::vector<std::pair<uint32_t, uint32_t>> rev;  // (target v, source u)
    for (size_t t = 0; t < nb; ++t)
      for (uint32_t v : fresh[t]) rev.push_back({v, uint32_t(order[b0 + t])});
    std::stable_sort(rev.begin(), rev.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
    std::vector<std::pair<size_t, size_t>> groups;
    for (size_t i = 0; i < rev.size();) {
      size_t j = i;
      while (j < rev.size() && rev[j].first == rev[i].first) ++j;
      groups.push_back({i, j});
      i = j;
    }
    std::vector<std::vector<uint32_t>> updated(groups.size());
    std::vector<char> changed(groups.size(), 0);
    parallel_for(0, groups.size(), threads, [&](size_t gi) {
      const uint32_t v = rev[groups[gi].first].first;
      const auto& cur = g[v];
      std::vector<uint32_t> add;
      for (size_t i = groups[gi].first; i < groups[gi].second; ++i) {
        const uint32_t u = rev[i].second;
        if (std::find(cur.begin(), cur.end(), u) == cur.end()) add.push_back(u);
      }
      if (add.empty()) return;
      changed[gi] = 1;
      if (cur.size() + add.size() <= R) {
        updated[gi] = cur;
        updated[gi].insert(updated[gi].end(), add.begin(), add.end());
      } else {
        std::vector<Pair> cand;
        const float* xv = X + size_t(v) * dim;
        for (uint32_t w : cur) cand.push_back({l2_ref(xv, X + size_t(w) * dim, dim), w});
        for (uint32_t w : add) cand.push_back({l2_ref(xv, X + size_t(w) * dim, dim), w});
        std::sort(cand.begin(), cand.end());
        updated[gi] = robust_prune(X, dim, v, cand, alpha, R);
      }
    });
    for (size_t gi = 0; gi < groups.size(); ++gi)
      if (changed[gi]) g[rev[groups[gi].first].first] = std::move(updated[gi]);
  }
}

// ----------------------------------------------------------------------------
// Vamana::knn (src/vamana/vamana.hh:57-452)
// ----------------------------------------------------------------------------

struct Index {
  uint32_t n, dim, R, bits, metric, medoid;
  const uint32_t* adj;      // n*R, kEmpty-filled
  const uint8_t* records;   // n*rec_size, reference layout
  uint32_t rec_size;
  const float* vecs;        // n*dim
  const float* P;           // dim*dim column-major
  const float* c_rot;       // dim
};

struct BeamEntry {  // VamanaCoroutine::BeamEntry (src/coroutine.hh:56-60)
  uint32_t id;
  float distance;
  bool expanded;
};

// insert_into_beam (src/vamana/vamana.hh:1014-1030).
void insert_into_beam(std::vector<BeamEntry>& beam, uint32_t id, float dist, uint32_t cap) {
  auto it = std::lower_bound(beam.begin(), beam.end(), dist,
                             [](const BeamEntry& e, float d) { return e.distance < d; });
  beam.insert(it, {id, dist, false});
  if (beam.size() > cap) beam.resize(cap);
}

struct KnnOut {
  std::vector<BeamEntry> beam;  // final beam, sorted
  uint32_t H = 0, E = 0, Cr = 0;
};

// mode 0 = rabitq_gpu, 1 = exact_gpu (src/common/configuration.hh:128-130).
KnnOut knn_one(const Index& ix, const float* q, uint32_t L, int mode, const float* qr_in, const float* f_in,
               bool sort_final = true) {
  KnnOut o;
  const bool rabitq = mode == 0;
  const uint32_t D = ix.dim;
  std::vector<float> qr(D);
  float f3[3] = {0, 0, 0};
  if (rabitq) {
    if (qr_in) {
      std::copy(qr_in, qr_in + D, qr.begin());
    } else {
      rotate(ix.P, q, D, qr.data());
    }
    if (f_in) {
      f3[0] = f_in[0];
      f3[1] = f_in[1];
      f3[2] = f_in[2];
    } else {
      query_factors(qr.data(), ix.c_rot, D, ix.bits, f3);
    }
  }
  const uint32_t m = ix.medoid;
  const float* xm = ix.vecs + size_t(m) * D;
  const float md = ix.metric == 1 ? seed_ip(q, xm, D) : seed_l2(q, xm, D);
  auto& beam = o.beam;
  beam.push_back({m, md, false});
  std::unordered_set<uint32_t> visited;
  visited.insert(m);
  const uint32_t cap = rabitq ? L + kRabitqSearchBeamSlack : L;
  std::vector<uint32_t> unvisited;
  std::vector<float> dists;
  for (;;) {
    int best = -1;
    float best_dist = std::numeric_limits<float>::max();
    for (int i = 0; i < int(beam.size()); ++i)
      if (!beam[i].expanded && beam[i].distance < best_dist) {
        best_dist = beam[i].distance;
        best = i;
      }
    if (best < 0) break;
    beam[best].expanded = true;
    ++o.H;
    const uint32_t* row = ix.adj + size_t(beam[best].id) * ix.R;
    unvisited.clear();
    for (uint32_t j = 0; j < ix.R; ++j) {
      const uint32_t nb = row[j];
      if (nb == kEmpty) continue;
      if (visited.insert(nb).second) unvisited.push_back(nb);
    }
    if (unvisited.empty()) continue;
    dists.resize(unvisited.size());
    for (size_t i = 0; i < unvisited.size(); ++i) {
      const uint32_t c = unvisited[i];
      dists[i] = rabitq ? rabitq_estimate_one(qr.data(), f3, ix.records + size_t(c) * ix.rec_size, D, ix.bits)
                        : l2_ref(q, ix.vecs + size_t(c) * D, D);
    }
    o.E += uint32_t(unvisited.size());
    for (size_t i = 0; i < unvisited.size(); ++i) insert_into_beam(beam, unvisited[i], dists[i], cap);
  }
  if (rabitq && !beam.empty()) {
    for (auto& e : beam) e.distance = l2_ref(q, ix.vecs + size_t(e.id) * D, D);
    o.Cr = uint32_t(beam.size());
  }
  if (sort_final)
    std::sort(beam.begin(), beam.end(), [](const BeamEntry& a, const BeamEntry& b) { return a.distance < b.distance; });
  return o;
}


// ----------------------------------------------------------------------------
// Online insert (src/vamana/vamana.hh:458-999)
// ----------------------------------------------------------------------------

// rabitq_quantize_single_kernel<4,B> (src/gpu/kernels/distance_kernels.cuh:376-464)
// on an already rotated vector: float arithmetic, lane t of the 4-lane tile
// takes dims j = t mod 4, tile sums by the butterfly, IEEE division and square
// root, nvcc's contractions (every `acc += a*b` is an fma; the double
// t_const*|o| + 1e-5 is a double fma).  The online insert quantizes with this
// kernel, not with the offline builder's routine.
void quantize_gpu_rotated(const float* r, const float* c, double tc, uint32_t dim, uint32_t bits, uint8_t* out) {
  const uint32_t packed = (bits * dim + 7) / 8;
  float l2p[4] = {0, 0, 0, 0};
  for (uint32_t j = 0; j < dim; ++j) {
    const float diff = r[j] - c[j];
    l2p[j & 3] = std::fmaf(diff, diff, l2p[j & 3]);
  }
  const float l2_sqr = tile4(l2p);
  const float l2_norm = std::sqrt(l2_sqr);
  std::vector<uint8_t> u(dim);
  float ipp[4] = {0, 0, 0, 0};
  const int top = 1 << (bits - 1);
  for (uint32_t j = 0; j < dim; ++j) {
    const float abs_o = std::fabs((r[j] - c[j]) / l2_norm);
    int val = static_cast<int>(std::fma(tc, static_cast<double>(abs_o), 1e-5));
    if (val >= top) val = top - 1;
    u[j] = static_cast<uint8_t>(val);
    ipp[j & 3] = std::fmaf(static_cast<float>(val) + 0.5f, abs_o, ipp[j & 3]);
  }
  const float ip_norm = tile4(ipp);
  const float ip_norm_inv = ip_norm == 0.0f ? 1.0f : 1.0f / ip_norm;
  const uint32_t mask = uint32_t(top) - 1u;
  for (uint32_t j = 0; j < dim; ++j) {
    if (r[j] - c[j] >= 0.0f)
      u[j] = static_cast<uint8_t>(u[j] + top);
    else
      u[j] = static_cast<uint8_t>((~u[j]) & mask);
  }
  const float cb = -(static_cast<float>(top) - 0.5f);
  float rx[4] = {0, 0, 0, 0}, cx[4] = {0, 0, 0, 0};
  for (uint32_t j = 0; j < dim; ++j) {
    const float residual = r[j] - c[j];
    const float xu_cb = static_cast<float>(u[j]) + cb;
    rx[j & 3] = std::fmaf(residual, xu_cb, rx[j & 3]);
    cx[j & 3] = std::fmaf(c[j], xu_cb, cx[j & 3]);
  }
  float ip_resi = tile4(rx);
  const float ip_cent = tile4(cx);
  if (ip_resi == 0.0f) ip_resi = std::numeric_limits<float>::max();
  const float add = l2_sqr + ((2.0f * l2_sqr) * ip_cent) / ip_resi;
  const float rescale = (ip_norm_inv * -2.0f) * l2_norm;
  const uint32_t per = 8 / bits;
  for (uint32_t b = 0; b < packed; ++b) {
    uint32_t v = 0;
    for (uint32_t k = 0; k < per && b * per + k < dim; ++k) v |= uint32_t(u[b * per + k]) << (k * bits);
    out[b] = static_cast<uint8_t>(v);
  }
  std::memcpy(out + packed, &add, 4);
  std::memcpy(out + packed + 4, &rescale, 4);
}

// robust_prune_kernel (src/gpu/kernels/distance_kernels.cuh:285-370): candidates
// sorted by distance from the source (position s holds original index
// order[s], or s); the nearest valid candidate is kept, and every later valid
// candidate p' with alpha * |p* - p'|^2 <= d(source, p') is dropped (the
// squared distance a sequential fma chain over the dims), until R are kept.
// Writes original indices; returns the count.
uint32_t robust_prune_gpu(const float* vecs, uint32_t vstride, const float* dists, const uint32_t* order, uint32_t n,
                          uint32_t dim, float alpha, uint32_t R, uint32_t* out) {
  if (n <= R) {
    for (uint32_t i = 0; i < n; ++i) out[i] = order ? order[i] : i;
    return n;
  }
  std::vector<char> valid(n, 1);
  uint32_t cnt = 0;
  for (uint32_t start = 0; start < n && cnt < R; ++start) {
    if (!valid[start]) continue;
    const uint32_t ps = order ? order[start] : start;
    out[cnt++] = ps;
    const float* pv = vecs + size_t(ps) * vstride;
    for (uint32_t i = start + 1; i < n; ++i) {
      if (!valid[i]) continue;
      const float* qv = vecs + size_t(order ? order[i] : i) * vstride;
      float d = 0.0f;
      for (uint32_t k = 0; k < dim; ++k) {
        const float diff = pv[k] - qv[k];
        d = std::fmaf(diff, diff, d);
      }
      if (alpha * d <= dists[i]) valid[i] = 0;
    }
  }
  return cnt;
}

// A mutable index with spare rows for inserts.
struct MutIndex {
  uint32_t n, cap, dim, R, bits, metric, medoid;
  uint32_t* adj;
  uint8_t* records;
  uint32_t rec_size;
  float* vecs;
  uint32_t* ids;
  const float* P;
  const float* c_rot;
  double tc;
};

// Appends slot `v`'s reverse edge to `nb` (vamana.hh:795-986): room -> append;
// full -> RobustPrune of nb's neighbours plus v from nb's vector, distances by
// batch_l2_squared_distance_kernel, ordered by (distance, position).
void reverse_edge(MutIndex& ix, uint32_t nb, uint32_t v, float alpha) {
  uint32_t* row = ix.adj + size_t(nb) * ix.R;
  uint32_t cnt = 0;
  while (cnt < ix.R && row[cnt] != kEmpty) ++cnt;
  if (cnt < ix.R) {
    row[cnt] = v;
    return;
  }
  std::vector<uint32_t> all(row, row + ix.R);
  all.push_back(v);
  const uint32_t n_all = uint32_t(all.size());
  const float* src = ix.vecs + size_t(nb) * ix.dim;
  std::vector<float> d(n_all);
  std::vector<float> cand(size_t(n_all) * ix.dim);
  for (uint32_t i = 0; i < n_all; ++i) {
    std::memcpy(&cand[size_t(i) * ix.dim], ix.vecs + size_t(all[i]) * ix.dim, size_t(ix.dim) * 4);
    d[i] = l2_ref(src, &cand[size_t(i) * ix.dim], ix.dim);
  }
  std::vector<uint32_t> order(n_all);
  for (uint32_t i = 0; i < n_all; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return d[a] < d[b]; });
  std::vector<float> sd(n_all);
  for (uint32_t i = 0; i < n_all; ++i) sd[i] = d[order[i]];
  std::vector<uint32_t> kept(ix.R);
  const uint32_t nk = robust_prune_gpu(cand.data(), ix.dim, sd.data(), order.data(), n_all, ix.dim, alpha, ix.R,
                                       kept.data());
  for (uint32_t i = 0; i < ix.R; ++i) row[i] = i < nk ? all[kept[i]] : kEmpty;
}

struct InsertCounts {
  uint64_t H = 0, E = 0, full_prunes = 0;
};

// One batch: every vector searches the graph as it stood at the start of the
// batch (beam search with exact distances, capacity L_c, vamana.hh:566-661),
// its final beam in beam order is pruned (vamana.hh:663-746), the new nodes
// are written, then reverse edges are added in insert order
// (vamana.hh:795-986).  An empty index first takes vector 0 as the medoid
// with no neighbours (vamana.hh:479-546).
void insert_batch(MutIndex& ix, const float* X, const uint32_t* new_ids, uint32_t B, uint32_t Lc, float alpha,
                  InsertCounts& cnt, int threads) {
  const uint32_t D = ix.dim;
  const uint32_t rs = ix.rec_size;
  auto write_node = [&](uint32_t slot, const float* x, uint32_t id, const uint32_t* nbrs, uint32_t nn) {
    std::memcpy(ix.vecs + size_t(slot) * D, x, size_t(D) * 4);
    ix.ids[slot] = id;
    std::vector<float> r(D);
    rotate(ix.P, x, D, r.data());
    quantize_gpu_rotated(r.data(), ix.c_rot, ix.tc, D, ix.bits, ix.records + size_t(slot) * rs);
    uint32_t* row = ix.adj + size_t(slot) * ix.R;
    for (uint32_t j = 0; j < ix.R; ++j) row[j] = j < nn ? nbrs[j] : kEmpty;
  };
  uint32_t first = 0;
  if (ix.n == 0 && B > 0) {
    write_node(0, X, new_ids[0], nullptr, 0);
    ix.medoid = 0;
    ix.n = 1;
    first = 1;
  }
  const uint32_t m = B - first;
  if (m == 0) return;
  const uint32_t n0 = ix.n;
  Index frozen{ix.n, D, ix.R, ix.bits, ix.metric, ix.medoid, ix.adj, ix.records, rs, ix.vecs, ix.P, ix.c_rot};
  std::vector<uint32_t> pruned(size_t(m) * ix.R, kEmpty), npr(m);
  std::vector<uint32_t> H(m), E(m);
  parallel_for(0, m, threads, [&](size_t i) {
    const KnnOut o = knn_one(frozen, X + size_t(first + i) * D, Lc, 1, nullptr, nullptr, false);
    H[i] = o.H;
    E[i] = o.E;
    const uint32_t nc = uint32_t(o.beam.size());
    std::vector<float> cv(size_t(nc) * D), cd(nc);
    for (uint32_t c = 0; c < nc; ++c) {
      std::memcpy(&cv[size_t(c) * D], ix.vecs + size_t(o.beam[c].id) * D, size_t(D) * 4);
      cd[c] = o.beam[c].distance;
    }
    std::vector<uint32_t> kept(ix.R);
    const uint32_t nk = robust_prune_gpu(cv.data(), D, cd.data(), nullptr, nc, D, alpha, ix.R, kept.data());
    npr[i] = nk;
    for (uint32_t j = 0; j < nk; ++j) pruned[size_t(i) * ix.R + j] = o.beam[kept[j]].id;
  });
  for (uint32_t i = 0; i < m; ++i) {
    write_node(n0 + i, X + size_t(first + i) * D, new_ids[first + i], &pruned[size_t(i) * ix.R], npr[i]);
    cnt.H += H[i];
    cnt.E += E[i];
  }
  ix.n = n0 + m;
  for (uint32_t i = 0; i < m; ++i)
    for (uint32_t j = 0; j < npr[i]; ++j) {
      const uint32_t nb = pruned[size_t(i) * ix.R + j];
      uint32_t c = 0;
      const uint32_t* row = ix.adj + size_t(nb) * ix.R;
      while (c < ix.R && row[c] != kEmpty) ++c;
      if (c == ix.R) ++cnt.full_prunes;
      reverse_edge(ix, nb, n0 + i, alpha);
    }
}

bool write_all(const std::string& path, const void* data, size_t bytes) {
  std::ofstream out(path, std::ios::binary);
  if (!out.good()) return false;
  out.write(static_cast<const char*>(data), std::streamsize(bytes));
  return out.good();
}

}  // namespace

// ============================================================================
// C ABI
// ============================================================================
extern "C" {

// --- distances and estimator ---
float orc_l2_ref(const float* q, const float* x, uint32_t dim) { return l2_ref(q, x, dim); }
float orc_seed_l2(const float* a, const float* b, uint32_t dim) { return seed_l2(a, b, dim); }
float orc_seed_ip(const float* a, const float* b, uint32_t dim) { return seed_ip(a, b, dim); }

void orc_l2_batch(const float* q, const float* cand, uint32_t n, uint32_t dim, float* out) {
  for (uint32_t i = 0; i < n; ++i) out[i] = l2_ref(q, cand + size_t(i) * dim, dim);
}

void orc_rotate(const float* P, const float* x, uint32_t dim, float* out) { rotate(P, x, dim, out); }

void orc_query_factors(const float* q_rot, const float* c_rot, uint32_t dim, uint32_t bits, float* f3) {
  query_factors(q_rot, c_rot, dim, bits, f3);
}

void orc_query_prepare(const float* q, const float* P, const float* c_rot, uint32_t dim, uint32_t bits,
                       float* q_rot, float* f3) {
  rotate(P, q, dim, q_rot);
  query_factors(q_rot, c_rot, dim, bits, f3);
}

void orc_rabitq_estimate(const float* q_rot, const float* f3, const uint8_t* records, uint32_t rec_stride,
                         uint32_t n, uint32_t dim, uint32_t bits, float* out) {
  for (uint32_t i = 0; i < n; ++i) out[i] = rabitq_estimate_one(q_rot, f3, records + size_t(i) * rec_stride, dim, bits);
}

// --- RaBitQ build side ---
double orc_best_rescale_factor(const float* abs_unit, size_t dim, size_t bits) {
  return best_rescale_factor(abs_unit, dim, bits);
}
double orc_t_const(size_t dim, size_t bits, uint64_t seed) { return t_const(dim, bits, seed); }
void orc_gaussian_matrix(uint32_t dim, int seed, double* out) { gaussian_matrix(dim, seed, out); }
void orc_rotation_matrix(uint32_t dim, int seed, float* P) { rotation_matrix(dim, seed, P); }
void orc_centroid(const float* X, size_t n, uint32_t dim, float* out) { centroid(X, n, dim, out); }

void orc_quantize_rotated(const float* x_rot, const float* c_rot, double tc, uint32_t dim, uint32_t bits,
                          uint8_t* out) {
  quantize_rotated(x_rot, c_rot, tc, dim, bits, out);
}

// Quantize n vectors: rotate with the canonical order, then rabitq_quantize_vector.
void orc_quantize_batch(const float* X, size_t n, uint32_t dim, uint32_t bits, const float* P, const float* c_rot,
                        double tc, uint8_t* out, uint32_t rec_size, int threads) {
  parallel_for(0, n, threads, [&](size_t i) {
    std::vector<float> r(dim);
    rotate(P, X + i * dim, dim, r.data());
    quantize_rotated(r.data(), c_rot, tc, dim, bits, out + i * rec_size);
  });
}

// --- builder ---
uint64_t orc_compute_medoid(const float* X, uint64_t n, uint32_t dim) { return compute_medoid(X, n, dim); }

void orc_random_init(uint64_t n, uint32_t R, uint64_t seed, uint32_t* adj) {
  std::vector<std::vector<uint32_t>> g;
  random_init(n, R, seed, g);
  for (size_t i = 0; i < n; ++i) {
    for (uint32_t j = 0; j < R; ++j) adj[i * R + j] = j < g[i].size() ? g[i][j] : kEmpty;
  }
}

void orc_insert_order(uint64_t n, uint64_t seed, uint32_t* order) {
  std::vector<size_t> o(n);
  std::iota(o.begin(), o.end(), 0);
  std::mt19937 rng(seed);
  std::shuffle(o.begin(), o.end(), rng);
  for (size_t i = 0; i < n; ++i) order[i] = uint32_t(o[i]);
}

// Beam search of the builder on a fixed graph; writes up to cap (dist, id) pairs.
uint32_t orc_build_beam_search(const float* X, uint64_t n, uint32_t dim, const uint32_t* adj, uint32_t R,
                               uint32_t medoid, const float* q, uint32_t L, float* out_d, uint32_t* out_id,
                               uint32_t cap) {
  std::vector<std::vector<uint32_t>> g(n);
  for (size_t i = 0; i < n; ++i)
    for (uint32_t j = 0; j < R; ++j)
      if (adj[i * R + j] != kEmpty) g[i].push_back(adj[i * R + j]);
  auto v = build_beam_search(g, X, dim, medoid, q, L);
  const uint32_t m = uint32_t(std::min<size_t>(v.size(), cap));
  for (uint32_t i = 0; i < m; ++i) {
    out_d[i] = v[i].first;
    out_id[i] = v[i].second;
  }
  return uint32_t(v.size());
}

uint32_t orc_robust_prune(const float* X, uint32_t dim, uint32_t source, const float* cand_d,
                          const uint32_t* cand_id, uint32_t n_cand, float alpha, uint32_t R, uint32_t* out) {
  std::vector<Pair> c(n_cand);
  for (uint32_t i = 0; i < n_cand; ++i) c[i] = {cand_d[i], cand_id[i]};
  auto s = robust_prune(X, dim, source, c, alpha, R);
  std::copy(s.begin(), s.end(), out);
  return uint32_t(s.size());
}

void orc_batch_schedule(uint64_t n, uint64_t cap, uint64_t* out_bounds, uint64_t* out_count) {
  auto s = batch_schedule(n, cap);
  *out_count = s.size();
  if (out_bounds)
    for (size_t i = 0; i < s.size(); ++i) out_bounds[i] = s[i].second;
}

// Builds the graph; adj_out is n*R with kEmpty fill.  Returns the medoid.
uint64_t orc_build_graph(const float* X, uint64_t n, uint32_t dim, uint32_t R, uint32_t L, float alpha,
                         uint64_t seed, uint64_t batch_cap, int threads, uint32_t* adj_out) {
  std::vector<std::vector<uint32_t>> g;
  size_t medoid = 0;
  build_graph(X, n, dim, R, L, alpha, seed, batch_cap, threads, g, medoid);
  for (size_t i = 0; i < n; ++i)
    for (uint32_t j = 0; j < R; ++j) adj_out[i * R + j] = j < g[i].size() ? g[i][j] : kEmpty;
  return medoid;
}

// --- shard writer (write_vamana_shards, tools/vamana_offline_builder.cc:1110-1267) ---
// Node i lands in shard i mod M at offset 16 + (i div M) * align8(node_size),
// because every shard starts at 16 and min_element picks the first minimum.
int orc_write_shards(const char* prefix, const float* X, uint64_t n, uint32_t dim, uint32_t R, uint32_t bits,
                     const uint32_t* adj, uint32_t medoid, const uint8_t* records, const float* P,
                     const float* c_rot, double tc, uint32_t M, uint32_t beam_width, double alpha, int ip) {
  const uint32_t rabitq_size = (bits * dim + 7) / 8 + 8;
  const size_t node_size = 8 + 8 + size_t(dim) * 4 + rabitq_size + size_t(R) * 8;
  const size_t aligned = (node_size + 7) & ~size_t(7);
  auto shard_of = [&](size_t i) { return uint32_t(i % M); };
  auto off_of = [&](size_t i) { return uint64_t(16 + (i / M) * aligned); };
  auto rptr = [&](size_t i) { return (uint64_t(shard_of(i)) << 48) | off_of(i); };
  std::vector<std::vector<uint8_t>> shards(M);
  for (uint32_t s = 0; s < M; ++s) {
    const size_t count = n / M + (s < n % M ? 1 : 0);
    const uint64_t sz = 16 + count * aligned;
    shards[s].assign(sz, 0);
    std::memcpy(shards[s].data(), &sz, 8);
  }
  const uint64_t mp = rptr(medoid);
  std::memcpy(shards[0].data() + 8, &mp, 8);
  for (size_t i = 0; i < n; ++i) {
    uint8_t* buf = shards[shard_of(i)].data() + off_of(i);
    uint64_t header = (i == medoid) ? 0b10000000000000000ull : 0;
    std::memcpy(buf, &header, 8);
    const uint32_t id = uint32_t(i);
    std::memcpy(buf + 8, &id, 4);
    uint8_t ec = 0;
    for (uint32_t j = 0; j < R; ++j)
      if (adj[i * R + j] != kEmpty) ++ec;
    buf[12] = ec;
    std::memcpy(buf + 16, X + i * dim, size_t(dim) * 4);
    std::memcpy(buf + 16 + size_t(dim) * 4, records + i * rabitq_size, rabitq_size);
    uint8_t* nb = buf + 16 + size_t(dim) * 4 + rabitq_size;
    uint32_t w = 0;
    for (uint32_t j = 0; j < R; ++j) {
      if (adj[i * R + j] == kEmpty) continue;
      const uint64_t p = rptr(adj[i * R + j]);
      std::memcpy(nb + size_t(w++) * 8, &p, 8);
    }
  }
  const std::string pre(prefix);
  for (uint32_t s = 0; s < M; ++s) {
    const std::string f = pre + "_node" + std::to_string(s + 1) + "_of" + std::to_string(M) + ".dat";
    if (!write_all(f, shards[s].data(), shards[s].size())) return -1;
  }
  {
    std::ofstream out(pre + ".rotation.bin", std::ios::binary);
    if (!out.good()) return -1;
    out.write(reinterpret_cast<const char*>(&dim), 4);
    out.write(reinterpret_cast<const char*>(P), std::streamsize(size_t(dim) * dim * 4));
    out.write(reinterpret_cast<const char*>(c_rot), std::streamsize(size_t(dim) * 4));
    out.write(reinterpret_cast<const char*>(&tc), 8);
    if (!out.good()) return -1;
  }
  {
    std::ofstream out(pre + ".meta.json");
    if (!out.good()) return -1;
    char buf[1024];
    std::snprintf(buf, sizeof(buf),
                  "{\n  \"R\": %u,\n  \"alpha\": %.15g,\n  \"beam_width\": %u,\n  \"beam_width_construction\": %u,\n"
                  "  \"dim\": %u,\n  \"distance\": \"%s\",\n  \"medoid\": {\n    \"memory_node\": %u,\n"
                  "    \"offset\": %llu\n  },\n  \"node_size\": %zu,\n  \"num_memory_nodes\": %u,\n"
                  "  \"num_vectors\": %llu,\n  \"rabitq_bits\": %u,\n  \"rabitq_size\": %u\n}\n",
                  R, alpha, beam_width, beam_width, dim, ip ? "ip" : "l2", uint32_t(mp >> 48),
                  (unsigned long long)(mp & 0xFFFFFFFFFFFFull), node_size, M, (unsigned long long)n, bits,
                  rabitq_size);
    out << buf;
    if (!out.good()) return -1;
  }
  return 0;
}

// --- knn ---
// counters: nq*4 = (H expansions, E estimates, C_r reranked rows, result count).
// beam_out_* (optional): nq*beam_cap final sorted beam ids/dists.
int orc_knn(uint32_t n, uint32_t dim, uint32_t R, uint32_t bits, uint32_t metric, uint32_t medoid,
            const uint32_t* adj, const uint8_t* records, uint32_t rec_size, const float* vecs, const float* P,
            const float* c_rot, const float* queries, uint32_t nq, uint32_t k, uint32_t beam_width, int mode,
            const float* q_rot_in, const float* f_in, uint32_t* out_ids, float* out_dist, uint32_t* counters,
            uint32_t* beam_out_ids, float* beam_out_dist, uint32_t beam_cap, int threads) {
  if (beam_width < k || k == 0) return -1;
  Index ix{n, dim, R, bits, metric, medoid, adj, records, rec_size, vecs, P, c_rot};
  parallel_for(0, nq, threads, [&](size_t qi) {
    const KnnOut o = knn_one(ix, queries + qi * dim, beam_width, mode, q_rot_in ? q_rot_in + qi * dim : nullptr,
                             f_in ? f_in + qi * 3 : nullptr);
    const uint32_t cnt = uint32_t(std::min<size_t>(k, o.beam.size()));
    for (uint32_t i = 0; i < k; ++i) {
      out_ids[qi * k + i] = i < cnt ? o.beam[i].id : kEmpty;
      out_dist[qi * k + i] = i < cnt ? o.beam[i].distance : std::numeric_limits<float>::infinity();
    }
    if (counters) {
      counters[qi * 4 + 0] = o.H;
      counters[qi * 4 + 1] = o.E;
      counters[qi * 4 + 2] = o.Cr;
      counters[qi * 4 + 3] = cnt;
    }
    if (beam_out_ids) {
      for (uint32_t i = 0; i < beam_cap; ++i) {
        beam_out_ids[qi * beam_cap + i] = i < o.beam.size() ? o.beam[i].id : kEmpty;
        beam_out_dist[qi * beam_cap + i] =
            i < o.beam.size() ? o.beam[i].distance : std::numeric_limits<float>::infinity();
      }
    }
  });
  return 0;
}


// --- online insert ---
void orc_quantize_gpu_rotated(const float* x_rot, const float* c_rot, double tc, uint32_t dim, uint32_t bits,
                              uint8_t* out) {
  quantize_gpu_rotated(x_rot, c_rot, tc, dim, bits, out);
}

uint32_t orc_robust_prune_gpu(const float* vecs, const float* dists, const uint32_t* order, uint32_t n, uint32_t dim,
                              float alpha, uint32_t R, uint32_t* out) {
  return robust_prune_gpu(vecs, dim, dists, order, n, dim, alpha, R, out);
}

// Inserts B vectors into an index held in caller arrays with room for `cap`
// rows; *n and *medoid are updated.  counts = {expansions, distances, full prunes}.
int orc_insert_batch(uint32_t* n, uint32_t cap, uint32_t dim, uint32_t R, uint32_t bits, uint32_t metric,
                     uint32_t* medoid, uint32_t* adj, uint8_t* records, uint32_t rec_size, float* vecs, uint32_t* ids,
                     const float* P, const float* c_rot, double t_const, const float* X, const uint32_t* new_ids,
                     uint32_t B, uint32_t Lc, float alpha, uint64_t* counts, int threads) {
  if (*n + uint64_t(B) > cap) return -1;
  MutIndex ix{*n, cap, dim, R, bits, metric, *medoid, adj, records, rec_size, vecs, ids, P, c_rot, t_const};
  InsertCounts c;
  insert_batch(ix, X, new_ids, B, Lc, alpha, c, threads);
  *n = ix.n;
  *medoid = ix.medoid;
  if (counts) {
    counts[0] = c.H;
    counts[1] = c.E;
    counts[2] = c.full_prunes;
  }
  return 0;
}

// make_deterministic_vector (test/src/main.cpp:37-51).
void orc_make_deterministic_vector(uint32_t seed, uint64_t dim, float* out) {
  uint64_t state = 1469598103934665603ull ^ static_cast<uint64_t>(seed);
  for (size_t i = 0; i < dim; ++i) {
    state ^= state >> 12;
    state ^= state << 25;
    state ^= state >> 27;
    const uint32_t value = static_cast<uint32_t>((state * 2685821657736338717ull) >> 32);
    out[i] = static_cast<float>(value % 10000) / 10000.0f;
  }
  out[seed % dim] += 4.0f;
  out[(seed * 17 + 3) % dim] += 1.0f;
}

}  // extern "C"
