// GPU offline builder: Vamana graph + RaBitQ records + shard files.
//
// It produces what tools/vamana_offline_builder.cc produces
// (build_vamana_graph :673-861, init_rabitq :978-1024, rabitq_quantize_vector
// :1030-1102, write_vamana_shards :1136-1267), in the batched, deterministic
// form the oracle restates: batches of the shuffled insertion order (sizes 1,
// 2, 4, ... up to a cap) each
//   (a) beam-search the graph frozen at batch start (one warp per node,
//       exact L2, beam sorted by (distance, id), capacity L; every computed
//       distance is kept: the visited set V);
//   (b) sort V plus the node's current neighbours by (distance, id), drop
//       adjacent duplicates and RobustPrune with build alpha 1.0 (one CTA per
//       node, bitonic sort in shared memory);
//   (c) replace the batch nodes' lists;
//   (d) add reverse edges grouped by target in batch order; a target that
//       would exceed R keeps RobustPrune(own list + additions).
// Distances use the reference GPU kernel's L2 order everywhere, so the graph
// equals the oracle's bit for bit.

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <numeric>
#include <queue>
#include <random>
#include <string>
#include <vector>

#include "device_math.cuh"
#include "internal.h"
#include "search.cuh"

using dvs::fail;

namespace dvs {
namespace {

constexpr uint32_t kFull = 0xFFFFFFFFu;
constexpr uint64_t kPadKey = ~uint64_t(0);

__device__ __forceinline__ uint64_t make_key(float d, uint32_t id) {
  uint32_t b = __float_as_uint(d == 0.f ? 0.f : d);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (uint64_t(b) << 32) | id;
}
__device__ __forceinline__ float key_dist(uint64_t k) {
  uint32_t b = uint32_t(k >> 32);
  b = (b & 0x80000000u) ? (b & 0x7FFFFFFFu) : ~b;
  return __uint_as_float(b);
}
__device__ __forceinline__ uint32_t key_id(uint64_t k) { return uint32_t(k); }

__device__ __forceinline__ bool tab_insert(uint32_t* tab, uint32_t cap, uint32_t id) {
  volatile uint32_t* vt = tab;
  uint32_t s = hash_slot(id, cap);
  for (uint32_t probe = 0; probe < cap; ++probe) {
    const uint32_t cur = vt[s];
    if (cur == id) return false;
    if (cur == kEmptySlot) {
      const uint32_t old = atomicCAS(tab + s, kEmptySlot, id);
      if (old == kEmptySlot) return true;
      if (old == id) return false;
    }
    s = (s + 1 == cap) ? 0 : s + 1;
  }
  return false;
}

__device__ __forceinline__ bool tab_contains(const uint32_t* tab, uint32_t cap, uint32_t id) {
  const volatile uint32_t* vt = tab;
  uint32_t s = hash_slot(id, cap);
  for (uint32_t probe = 0; probe < cap; ++probe) {
    const uint32_t cur = vt[s];
    if (cur == id) return true;
    if (cur == kEmptySlot) return false;
    s = (s + 1 == cap) ? 0 : s + 1;
  }
  return false;
}

struct BuildSearchArgs {
  const float* vecs = nullptr;
  const uint32_t* adj = nullptr;
  const uint32_t* nodes = nullptr;  // batch node ids
  uint64_t* seg = nullptr;          // nb * seg_cap keys
  uint32_t* seg_count = nullptr;
  uint32_t* work = nullptr;         // [0] next, [1] error bits
  uint32_t* ovf = nullptr;
  uint32_t vec_stride = 0, dim = 0, R = 0, medoid = 0, nb = 0, L = 0, seg_cap = 0;
  uint32_t hcap = 0, hlimit = 0, ovf_cap = 0, ovf_limit = 0, cap_pad = 0;
};

__host__ __device__ inline uint32_t build_warp_words(uint32_t cap_pad, uint32_t dim_pad, uint32_t hcap) {
  // two beam buffers of (u64 key + u32 flag), the query row, candidate ids and keys, the visited table
  return 2 * (3 * cap_pad) + dim_pad + 64 + 128 + hcap;
}

// (a) beam_search of the builder (tools/vamana_offline_builder.cc:523-625).
__global__ void __launch_bounds__(256) build_search_kernel(const BuildSearchArgs a) {
  extern __shared__ __align__(16) uint32_t smem[];
  const uint32_t lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const uint32_t dim_pad = a.vec_stride;
  uint32_t* base = smem + size_t(wib) * build_warp_words(a.cap_pad, dim_pad, a.hcap);
  uint64_t* bkA = reinterpret_cast<uint64_t*>(base);
  uint64_t* bkB = reinterpret_cast<uint64_t*>(base + 2 * a.cap_pad);
  uint32_t* bfA = base + 4 * a.cap_pad;
  uint32_t* bfB = base + 5 * a.cap_pad;
  float* qv = reinterpret_cast<float*>(base + 6 * a.cap_pad);
  uint32_t* cid = base + 6 * a.cap_pad + dim_pad;
  uint64_t* ckey = reinterpret_cast<uint64_t*>(cid + 64);
  uint32_t* htab = cid + 64 + 128;
  const uint32_t warp_slot = blockIdx.x * (blockDim.x >> 5) + wib;
  uint32_t* gtab = a.ovf + size_t(warp_slot) * a.ovf_cap;
  const uint32_t dim = a.dim, R = a.R, L = a.L;

  for (;;) {
    uint32_t t = 0;
    if (lane == 0) t = atomicAdd(a.work, 1u);
    t = __shfl_sync(kFull, t, 0);
    if (t >= a.nb) break;
    const uint32_t u = a.nodes[t];
    uint64_t* seg = a.seg + size_t(t) * a.seg_cap;
    for (uint32_t j = lane; j < dim_pad; j += 32) qv[j] = a.vecs[size_t(u) * a.vec_stride + j];
    {
      uint4* h4 = reinterpret_cast<uint4*>(htab);
      const uint4 e = make_uint4(kEmptySlot, kEmptySlot, kEmptySlot, kEmptySlot);
      for (uint32_t j = lane; j < (a.hcap >> 2); j += 32) h4[j] = e;
    }
    __syncwarp();
    // medoid seed: l2 in the reference kernel's order
    float part = l2_quad_partial(qv, a.vecs + size_t(a.medoid) * a.vec_stride, dim, lane & 3);
    const float md = quad_butterfly(part);
    if (lane == 0) {
      bkA[0] = make_key(md, a.medoid);
      bfA[0] = 0;
      htab[hash_slot(a.medoid, a.hcap)] = a.medoid;
      seg[0] = make_key(md, a.medoid);
    }
    __syncwarp();
    uint64_t* bk = bkA;
    uint32_t* bf = bfA;
    uint64_t* bko = bkB;
    uint32_t* bfo = bfB;
    uint32_t nb = 1, hcount = 1, gcount = 0, count = 1, err = 0;
    bool overflow = false;
    for (;;) {
      int best = -1;
      for (uint32_t b = 0; b < nb; b += 32) {
        const uint32_t p = b + lane;
        const uint32_t m = __ballot_sync(kFull, p < nb && bf[p] == 0);
        if (m) {
          best = int(b + __ffs(m) - 1);
          break;
        }
      }
      if (best < 0) break;
      const uint32_t x = key_id(bk[best]);
      __syncwarp();
      if (lane == 0) bf[best] = 1;
      uint32_t nbr[2];
      for (int s = 0; s < 2; ++s) {
        const uint32_t j = lane + 32u * s;
        nbr[s] = j < R ? __ldg(a.adj + size_t(x) * R + j) : kEmptySlot;
      }
      uint32_t m = 0;
      for (int s = 0; s < 2; ++s) {
        const uint32_t peers = __match_any_sync(kFull, nbr[s]);
        const bool first = nbr[s] != kEmptySlot && (peers & lanemask_lt()) == 0;
        if (!overflow && hcount + 32 > a.hlimit) {
          overflow = true;
          uint4* g4 = reinterpret_cast<uint4*>(gtab);
          const uint4 e = make_uint4(kEmptySlot, kEmptySlot, kEmptySlot, kEmptySlot);
          for (uint32_t j = lane; j < (a.ovf_cap >> 2); j += 32) g4[j] = e;
          __syncwarp();
        }
        if (overflow && gcount + 32 > a.ovf_limit) err |= kErrCapacity;
        if (err) break;
        bool fresh = false;
        if (first) {
          if (!overflow)
            fresh = tab_insert(htab, a.hcap, nbr[s]);
          else
            fresh = !tab_contains(htab, a.hcap, nbr[s]) && tab_insert(gtab, a.ovf_cap, nbr[s]);
        }
        const uint32_t bal = __ballot_sync(kFull, fresh);
        if (fresh) cid[m + __popc(bal & lanemask_lt())] = nbr[s];
        const uint32_t cnt = __popc(bal);
        m += cnt;
        if (overflow)
          gcount += cnt;
        else
          hcount += cnt;
        __syncwarp();
      }
      if (err) break;
      if (m == 0) continue;
      if (count + m > a.seg_cap) {
        err |= kErrCapacity;
        break;
      }
      // exact distances, 4 lanes per row
      for (uint32_t r0 = 0; r0 < m; r0 += 8) {
        const uint32_t i = r0 + (lane >> 2);
        float p2 = 0.f;
        if (i < m) p2 = l2_quad_partial(qv, a.vecs + size_t(cid[i]) * a.vec_stride, dim, lane & 3);
        const float tot = quad_butterfly(p2);
        if (i < m && (lane & 3) == 0) ckey[i] = make_key(tot, cid[i]);
      }
      __syncwarp();
      for (uint32_t i = lane; i < m; i += 32) seg[count + i] = ckey[i];
      count += m;
      // merge (keys are unique): beam sorted by (distance, id), capacity L
      const uint32_t nb_new = min(L, nb + m);
      for (uint32_t i = lane; i < m; i += 32) {
        const uint64_t k = ckey[i];
        uint32_t r = 0;
        for (uint32_t j = 0; j < m; ++j) r += ckey[j] < k;
        if (r >= L) continue;
        uint32_t lo = 0, hi = nb;
        while (lo < hi) {
          const uint32_t mid = (lo + hi) >> 1;
          if (bk[mid] < k)
            lo = mid + 1;
          else
            hi = mid;
        }
        const uint32_t pos = r + lo;
        if (pos < L) {
          bko[pos] = k;
          bfo[pos] = 0;
        }
      }
      for (uint32_t p = lane; p < nb; p += 32) {
        const uint64_t k = bk[p];
        uint32_t c = 0;
        for (uint32_t j = 0; j < m; ++j) c += ckey[j] < k;
        const uint32_t pos = p + c;
        if (pos < L) {
          bko[pos] = k;
          bfo[pos] = bf[p];
        }
      }
      __syncwarp();
      uint64_t* tk = bk;
      bk = bko;
      bko = tk;
      uint32_t* tf = bf;
      bf = bfo;
      bfo = tf;
      nb = nb_new;
    }
    // the node's current neighbours join the candidates (:742-748)
    if (!err) {
      uint32_t own[2];
      for (int s = 0; s < 2; ++s) {
        const uint32_t j = lane + 32u * s;
        own[s] = j < R ? a.adj[size_t(u) * R + j] : kEmptySlot;
      }
      uint32_t deg = 0;
      for (int s = 0; s < 2; ++s) deg += __popc(__ballot_sync(kFull, own[s] != kEmptySlot));
      if (count + deg > a.seg_cap) {
        err |= kErrCapacity;
      } else {
        for (int s = 0; s < 2; ++s) {
          const uint32_t bal = __ballot_sync(kFull, own[s] != kEmptySlot);
          if (own[s] != kEmptySlot) cid[__popc(bal & lanemask_lt())] = own[s];
          const uint32_t c2 = __popc(bal);
          __syncwarp();
          for (uint32_t r0 = 0; r0 < c2; r0 += 8) {
            const uint32_t i = r0 + (lane >> 2);
            float p2 = 0.f;
            if (i < c2) p2 = l2_quad_partial(qv, a.vecs + size_t(cid[i]) * a.vec_stride, dim, lane & 3);
            const float tot = quad_butterfly(p2);
            if (i < c2 && (lane & 3) == 0) seg[count + i] = make_key(tot, cid[i]);
          }
          count += c2;
          __syncwarp();
        }
      }
    }
    if (lane == 0) {
      a.seg_count[t] = err ? 0u : count;
      if (err) atomicOr(a.work + 1, err);
    }
    __syncwarp();
  }
}

// Bitonic sort of P (a power of two) keys in shared memory by the whole block.
__device__ void block_bitonic_sort(uint64_t* keys, uint32_t P) {
  for (uint32_t k = 2; k <= P; k <<= 1) {
    for (uint32_t j = k >> 1; j > 0; j >>= 1) {
      for (uint32_t i = threadIdx.x; i < P; i += blockDim.x) {
        const uint32_t ixj = i ^ j;
        if (ixj > i) {
          const uint64_t x = keys[i], y = keys[ixj];
          const bool up = (i & k) == 0;
          if ((x > y) == up) {
            keys[i] = y;
            keys[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
}

// RobustPrune (tools/vamana_offline_builder.cc:634-663) over `cnt` sorted keys,
// by the whole block: every thread tests one candidate of a chunk against the
// neighbours selected before the chunk; warp 0 then walks the chunk in order
// and tests the survivors against the neighbours selected inside the chunk.
// With `dedupe`, a key whose id equals its predecessor's is dropped first
// (std::unique on the sorted candidates, :750-752).  Returns |selected|.
__device__ uint32_t block_robust_prune(const uint64_t* keys, uint32_t cnt, uint32_t source, bool dedupe,
                                       const float* vecs, uint32_t vs, uint32_t dim, float alpha, uint32_t R,
                                       uint32_t* sel, uint8_t* pruned, uint32_t* state) {
  const uint32_t tid = threadIdx.x, lane = tid & 31;
  if (tid == 0) {
    state[0] = 0;  // selected
    state[1] = 0;  // done
  }
  __syncthreads();
  for (uint32_t c0 = 0; c0 < cnt; c0 += blockDim.x) {
    const uint32_t nsel0 = state[0];
    if (state[1]) break;
    const uint32_t i = c0 + tid;
    bool p = true;
    if (i < cnt) {
      const uint64_t k = keys[i];
      const uint32_t id = key_id(k);
      p = id == source || (dedupe && i > 0 && key_id(keys[i - 1]) == id);
      if (!p) {
        const float cd = key_dist(k);
        const float* xc = vecs + size_t(id) * vs;
        for (uint32_t s = 0; s < nsel0; ++s) {
          const float d = l2_single(vecs + size_t(sel[s]) * vs, xc, dim);
          if (__fmul_rn(alpha, d) <= cd) {
            p = true;
            break;
          }
        }
      }
    }
    pruned[tid] = p ? 1 : 0;
    __syncthreads();
    if (tid < 32) {
      uint32_t nsel = nsel0;
      const uint32_t len = min(blockDim.x, cnt - c0);
      for (uint32_t j = 0; j < len && nsel < R; ++j) {
        if (pruned[j]) continue;
        const uint64_t k = keys[c0 + j];
        const uint32_t id = key_id(k);
        const float cd = key_dist(k);
        bool pr = false;
        for (uint32_t s = nsel0; s < nsel && !pr; ++s) {
          const float part = l2_quad_partial(vecs + size_t(sel[s]) * vs, vecs + size_t(id) * vs, dim, lane & 3);
          const float d = quad_butterfly(part);
          pr = __fmul_rn(alpha, d) <= cd;
        }
        if (!pr) {
          if (lane == 0) sel[nsel] = id;
          ++nsel;
          __syncwarp();
        }
      }
      if (lane == 0) {
        state[0] = nsel;
        if (nsel >= R) state[1] = 1;
      }
    }
    __syncthreads();
  }
  return state[0];
}

struct PruneArgs {
  const float* vecs = nullptr;
  const uint32_t* nodes = nullptr;
  const uint64_t* seg = nullptr;
  const uint32_t* seg_count = nullptr;
  uint32_t* new_adj = nullptr;  // nb * R
  uint32_t vec_stride = 0, dim = 0, R = 0, seg_cap = 0, sort_cap = 0;
  float alpha = 1.f;
};

// (b) one block per batch node.
__global__ void __launch_bounds__(512) prune_kernel(const PruneArgs a) {
  extern __shared__ __align__(16) uint64_t keys[];
  __shared__ uint32_t sel[64];
  __shared__ uint8_t pruned[512];
  __shared__ uint32_t state[2];
  const uint32_t t = blockIdx.x;
  const uint32_t cnt = a.seg_count[t];
  uint32_t P = 2;
  while (P < cnt) P <<= 1;
  for (uint32_t i = threadIdx.x; i < P; i += blockDim.x) keys[i] = i < cnt ? a.seg[size_t(t) * a.seg_cap + i] : kPadKey;
  __syncthreads();
  block_bitonic_sort(keys, P);
  const uint32_t ns = block_robust_prune(keys, cnt, a.nodes[t], true, a.vecs, a.vec_stride, a.dim, a.alpha, a.R, sel,
                                         pruned, state);
  for (uint32_t j = threadIdx.x; j < a.R; j += blockDim.x) a.new_adj[size_t(t) * a.R + j] = j < ns ? sel[j] : kEmptySlot;
}

// (c) replace the batch nodes' lists.
__global__ void apply_kernel(uint32_t* adj, const uint32_t* nodes, const uint32_t* new_adj, uint32_t nb, uint32_t R) {
  const uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= uint64_t(nb) * R) return;
  const uint32_t t = uint32_t(i / R), j = uint32_t(i % R);
  adj[size_t(nodes[t]) * R + j] = new_adj[i];
}

struct ReverseArgs {
  const float* vecs = nullptr;
  uint32_t* adj = nullptr;
  const uint32_t* targets = nullptr;  // G targets
  const uint32_t* offsets = nullptr;  // G + 1
  const uint32_t* members = nullptr;  // sources in batch order
  uint32_t vec_stride = 0, dim = 0, R = 0;
  uint32_t key_cap = 0;               // keys the dynamic shared memory holds before the additions list
  float alpha = 1.f;
};

// (d) one block per reverse-edge target (tools/vamana_offline_builder.cc:762-800, batched).
__global__ void __launch_bounds__(256) reverse_kernel(const ReverseArgs a) {
  extern __shared__ __align__(16) uint64_t keys[];
  __shared__ uint32_t cur[64];
  __shared__ uint32_t sel[64];
  __shared__ uint8_t pruned[256];
  __shared__ uint32_t state[4];
  const uint32_t g = blockIdx.x;
  const uint32_t v = a.targets[g];
  const uint32_t m0 = a.offsets[g], m1 = a.offsets[g + 1];
  const uint32_t R = a.R;
  if (threadIdx.x < 64) cur[threadIdx.x] = threadIdx.x < R ? a.adj[size_t(v) * R + threadIdx.x] : kEmptySlot;
  if (threadIdx.x == 0) state[2] = 0;
  __syncthreads();
  uint32_t deg = 0;
  for (uint32_t j = 0; j < R; ++j) deg += cur[j] != kEmptySlot;
  // additions not already present, in batch order, staged past the key area
  uint32_t* add = reinterpret_cast<uint32_t*>(keys + a.key_cap);
  if (threadIdx.x == 0) {
    uint32_t na = 0;
    for (uint32_t i = m0; i < m1; ++i) {
      const uint32_t u = a.members[i];
      bool present = false;
      for (uint32_t j = 0; j < deg; ++j) present |= cur[j] == u;
      if (!present) add[na++] = u;
    }
    state[2] = na;
  }
  __syncthreads();
  const uint32_t na = state[2];
  if (na == 0) return;
  if (deg + na <= R) {
    for (uint32_t i = threadIdx.x; i < na; i += blockDim.x) a.adj[size_t(v) * R + deg + i] = add[i];
    return;
  }
  const uint32_t cnt = deg + na;
  uint32_t P = 2;
  while (P < cnt) P <<= 1;
  const float* xv = a.vecs + size_t(v) * a.vec_stride;
  for (uint32_t i = threadIdx.x; i < P; i += blockDim.x) {
    uint64_t k = kPadKey;
    if (i < cnt) {
      const uint32_t w = i < deg ? cur[i] : add[i - deg];
      k = make_key(l2_single(xv, a.vecs + size_t(w) * a.vec_stride, a.dim), w);
    }
    keys[i] = k;
  }
  __syncthreads();
  block_bitonic_sort(keys, P);
  const uint32_t ns = block_robust_prune(keys, cnt, v, false, a.vecs, a.vec_stride, a.dim, a.alpha, R, sel, pruned,
                                         state);
  __syncthreads();
  for (uint32_t j = threadIdx.x; j < R; j += blockDim.x) a.adj[size_t(v) * R + j] = j < ns ? sel[j] : kEmptySlot;
}

// RaBitQ records: rotate each vector in the canonical order (thread per output
// dim) and quantize it as rabitq_quantize_vector does, on one thread, in the
// written order (tools/vamana_offline_builder.cc:1030-1102).
__global__ void __launch_bounds__(128) quantize_kernel(const float* __restrict__ X, uint32_t x_stride,
                                                       const float* __restrict__ P, const float* __restrict__ c_rot,
                                                       double tc, uint32_t dim, uint32_t bits, uint32_t n,
                                                       uint8_t* __restrict__ out, uint32_t rs) {
  extern __shared__ float sh[];
  float* xs = sh;
  float* rot = sh + dim;
  uint8_t* qv = reinterpret_cast<uint8_t*>(sh + 2 * dim);
  for (uint32_t v = blockIdx.x; v < n; v += gridDim.x) {
    for (uint32_t j = threadIdx.x; j < dim; j += blockDim.x) xs[j] = X[size_t(v) * x_stride + j];
    __syncthreads();
    for (uint32_t j = threadIdx.x; j < dim; j += blockDim.x) {
      const float* col = P + size_t(j) * dim;
      float acc = 0.f;
      for (uint32_t i = 0; i < dim; ++i) acc = __fmaf_rn(__ldg(col + i), xs[i], acc);
      rot[j] = __fsub_rn(acc, c_rot[j]);  // delta
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      const double kEps = 1e-5;
      const uint32_t packed = (bits * dim + 7) / 8;
      float l2_sqr = 0.f;
      for (uint32_t i = 0; i < dim; ++i) l2_sqr = __fadd_rn(l2_sqr, __fmul_rn(rot[i], rot[i]));
      const float l2_norm = __fsqrt_rn(l2_sqr);
      const uint32_t cap = (1u << (bits - 1)) - 1u;
      float ip_norm = 0.f;
      for (uint32_t i = 0; i < dim; ++i) {
        const float abs_o = l2_norm > 0.f ? fabsf(__fdiv_rn(rot[i], l2_norm)) : 0.f;
        int val = int(__dadd_rn(__dmul_rn(tc, double(abs_o)), kEps));
        if (val >= int(1u << (bits - 1))) val = int(cap);
        qv[i] = uint8_t(val);
        ip_norm = __fadd_rn(ip_norm, __fmul_rn(__fadd_rn(float(val), 0.5f), abs_o));
      }
      const float ip_norm_inv = ip_norm == 0.f ? 1.f : __fdiv_rn(1.f, ip_norm);
      for (uint32_t i = 0; i < dim; ++i)
        qv[i] = rot[i] >= 0.f ? uint8_t(qv[i] + (1u << (bits - 1))) : uint8_t((~qv[i]) & cap);
      uint8_t* o = out + size_t(v) * rs;
      for (uint32_t b = 0; b < packed; ++b) o[b] = 0;
      for (uint32_t i = 0; i < dim; ++i) {
        const uint32_t bit_idx = i * bits, byte_idx = bit_idx / 8, bit_off = bit_idx % 8;
        o[byte_idx] |= uint8_t(qv[i] << bit_off);
        if (bit_off + bits > 8 && byte_idx + 1 < packed) o[byte_idx + 1] |= uint8_t(qv[i] >> (8 - bit_off));
      }
      const float cb = -(float(1u << (bits - 1)) - 0.5f);
      float ip_resi = 0.f, ip_cent = 0.f;
      for (uint32_t i = 0; i < dim; ++i) {
        const float xu_cb = __fadd_rn(float(qv[i]), cb);
        ip_resi = __fadd_rn(ip_resi, __fmul_rn(rot[i], xu_cb));
        ip_cent = __fadd_rn(ip_cent, __fmul_rn(c_rot[i], xu_cb));
      }
      if (ip_resi == 0.f) ip_resi = __int_as_float(0x7F800000);
      const float add_f = __fadd_rn(l2_sqr, __fdiv_rn(__fmul_rn(__fmul_rn(2.0f, l2_sqr), ip_cent), ip_resi));
      const float rescale_f = __fmul_rn(__fmul_rn(ip_norm_inv, -2.0f), l2_norm);
      const uint32_t ab = __float_as_uint(add_f), rb = __float_as_uint(rescale_f);
      for (int b = 0; b < 4; ++b) {
        o[packed + b] = uint8_t(ab >> (8 * b));
        o[packed + 4 + b] = uint8_t(rb >> (8 * b));
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

float host_l2_ref(const float* q, const float* x, uint32_t dim) {
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t n4 = dim / 4;
  for (uint32_t i = 0; i < n4; ++i)
    for (uint32_t k = 0; k < 4; ++k) {
      const float d = q[4 * i + k] - x[4 * i + k];
      s[i & 3] = std::fmaf(d, d, s[i & 3]);
    }
  for (uint32_t i = n4 * 4; i < dim; ++i) {
    const float d = q[i] - x[i];
    s[(i - n4 * 4) & 3] = std::fmaf(d, d, s[(i - n4 * 4) & 3]);
  }
  return (s[0] + s[2]) + (s[1] + s[3]);
}

constexpr float kTightStart[9] = {0.0f, 0.15f, 0.20f, 0.52f, 0.59f, 0.71f, 0.75f, 0.77f, 0.81f};

// best_rescale_factor / get_const_scaling_factors (tools/vamana_offline_builder.cc:889-973).
double best_rescale_factor(const float* o, size_t dim, size_t bits) {
  const double kEps = 1e-5;
  const double max_o = *std::max_element(o, o + dim);
  if (max_o <= 0.0) return 0.0;
  const double t_end = double(((1u << bits) - 1u) + 10) / max_o;
  const double t_start = t_end * kTightStart[bits];
  std::vector<int> cur(dim);
  double den = double(dim) * 0.25, num = 0.0;
  for (size_t i = 0; i < dim; ++i) {
    const int c = int((t_start * o[i]) + kEps);
    cur[i] = c;
    den += double(c) * c + c;
    num += (double(c) + 0.5) * o[i];
  }
  std::priority_queue<std::pair<double, size_t>, std::vector<std::pair<double, size_t>>, std::greater<>> pq;
  for (size_t i = 0; i < dim; ++i)
    if (o[i] > 0.0f) pq.emplace(double(cur[i] + 1) / o[i], i);
  double max_ip = 0.0, best_t = 0.0;
  while (!pq.empty()) {
    const auto [ct, id] = pq.top();
    pq.pop();
    const int u = ++cur[id];
    den += 2.0 * u;
    num += o[id];
    const double ip = num / std::sqrt(den);
    if (ip > max_ip) {
      max_ip = ip;
      best_t = ct;
    }
    if (u < int((1u << bits) - 1u)) {
      const double nt = double(u + 1) / o[id];
      if (nt < t_end) pq.emplace(nt, id);
    }
  }
  return best_t;
}

double t_const(size_t dim, size_t bits, uint64_t seed) {
  std::mt19937_64 rng(seed);
  std::normal_distribution<float> normal(0.0f, 1.0f);
  std::vector<float> s(dim), a(dim);
  double total = 0.0;
  for (size_t k = 0; k < 1000; ++k) {
    double ns = 0.0;
    for (size_t d = 0; d < dim; ++d) {
      s[d] = normal(rng);
      ns += double(s[d]) * s[d];
    }
    const double nrm = std::sqrt(ns);
    const double inv = nrm > 0.0 ? 1.0 / nrm : 0.0;
    for (size_t d = 0; d < dim; ++d) a[d] = std::fabs(float(s[d] * inv));
    total += best_rescale_factor(a.data(), dim, bits);
  }
  return total / 1000.0;
}

// P of init_rabitq: Householder QR of a mt19937(seed) Gaussian matrix (filled
// row by row), columns negated where R(i,i) < 0; double precision, then float.
void rotation_matrix(uint32_t dim, int seed, std::vector<float>& P) {
  const size_t D = dim;
  std::vector<double> A(D * D), A0;
  {
    std::mt19937 rng(seed);
    std::normal_distribution<float> normal(0.0f, 1.0f);
    for (size_t i = 0; i < D; ++i)
      for (size_t j = 0; j < D; ++j) A[i + j * D] = normal(rng);
  }
  A0 = A;
  std::vector<std::vector<double>> vs(D);
  for (size_t k = 0; k < D; ++k) {
    double nrm = 0.0;
    for (size_t i = k; i < D; ++i) nrm += A[i + k * D] * A[i + k * D];
    nrm = std::sqrt(nrm);
    const double alpha = A[k + k * D] >= 0 ? -nrm : nrm;
    std::vector<double> v(D - k);
    for (size_t i = k; i < D; ++i) v[i - k] = A[i + k * D];
    v[0] -= alpha;
    double vn = 0.0;
    for (double x : v) vn += x * x;
    vn = std::sqrt(vn);
    if (vn > 0) {
      for (double& x : v) x /= vn;
      for (size_t c = k; c < D; ++c) {
        double dot = 0.0;
        for (size_t i = k; i < D; ++i) dot += v[i - k] * A[i + c * D];
        for (size_t i = k; i < D; ++i) A[i + c * D] -= 2.0 * v[i - k] * dot;
      }
    }
    vs[k] = std::move(v);
  }
  std::vector<double> Q(D * D, 0.0);
  for (size_t i = 0; i < D; ++i) Q[i + i * D] = 1.0;
  for (size_t kk = D; kk-- > 0;) {
    const auto& v = vs[kk];
    for (size_t c = 0; c < D; ++c) {
      double dot = 0.0;
      for (size_t i = kk; i < D; ++i) dot += v[i - kk] * Q[i + c * D];
      for (size_t i = kk; i < D; ++i) Q[i + c * D] -= 2.0 * v[i - kk] * dot;
    }
  }
  P.resize(D * D);
  for (size_t c = 0; c < D; ++c) {
    double r = 0.0;
    for (size_t i = 0; i < D; ++i) r += Q[i + c * D] * A0[i + c * D];
    const double sg = r < 0.0 ? -1.0 : 1.0;
    for (size_t i = 0; i < D; ++i) P[i + c * D] = float(sg * Q[i + c * D]);
  }
}

#define DVS_CUDA(call)                                                                             \
  do {                                                                                             \
    const cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess) {                                                                       \
      return fail(e_ == cudaErrorMemoryAllocation ? DVS_ERR_OOM : DVS_ERR_CUDA,                    \
                  std::string(#call) + ": " + cudaGetErrorString(e_));                             \
    }                                                                                              \
  } while (0)

template <class T>
struct DevBuf {
  T* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  cudaError_t alloc(size_t n) {
    if (p) cudaFree(p);
    p = nullptr;
    return cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T));
  }
};

}  // namespace
}  // namespace dvs

extern "C" {

dvs_status dvs_build_index(const dvs_build_params* bp, const float* h_vecs, uint64_t n, uint32_t dim,
                           dvs_build_stats* stats) {
  using namespace dvs;
  if (!bp || !h_vecs) return fail(DVS_ERR_ARG, "null argument");
  if (n < 2 || n >= (1ull << 31)) return fail(DVS_ERR_ARG, "need 2 <= n < 2^31 vectors");
  if (dim == 0 || dim > 4096) return fail(DVS_ERR_DIM, "dim must be in 1..4096");
  const uint32_t R = bp->R, L = bp->beam_width, bits = bp->rabitq_bits;
  if (R == 0 || R > 64) return fail(DVS_ERR_ARG, "R must be in 1..64 for the GPU builder");
  if (L == 0 || L > 1024) return fail(DVS_ERR_ARG, "beam_width must be in 1..1024 for the GPU builder");
  if (bits != 1 && bits != 2 && bits != 4 && bits != 8) return fail(DVS_ERR_BITS, "rabitq_bits must be 1, 2, 4, or 8");
  // An inner-product index (metadata "distance": "ip", searched with the
  // 1 - dot medoid seed) is built with L2 graph distances.  For unit-norm
  // vectors, the configuration the reference's IP mode serves, 1 - dot equals
  // half the squared L2 distance: every ranking, the medoid and RobustPrune's
  // alpha test (both sides scale by 1/2) are the same, up to rounding.
  if (bp->metric != DVS_METRIC_L2 && bp->metric != DVS_METRIC_IP) return fail(DVS_ERR_ARG, "metric must be l2 or ip");
  for (uint64_t i = 0; i < n * dim; ++i)
    if (!std::isfinite(h_vecs[i])) return fail(DVS_ERR_ARG, "input vectors contain a non-finite value");
  if (stats) *stats = dvs_build_stats{};
  DVS_CUDA(cudaSetDevice(bp->device));
  cudaEvent_t e0, e1;
  DVS_CUDA(cudaEventCreate(&e0));
  DVS_CUDA(cudaEventCreate(&e1));
  DVS_CUDA(cudaEventRecord(e0));
  const size_t seed = bp->seed == -1 ? std::random_device{}() : size_t(bp->seed);
  const uint32_t vs = (dim + 3) / 4 * 4;
  const float alpha_build = 1.0f;  // tools/vamana_offline_builder.cc:723

  // ---- medoid (compute_medoid, :473-507) ----
  uint32_t medoid = 0;
  {
    const size_t ss = std::min<size_t>(n, 10000);
    std::vector<size_t> idx(n);
    std::iota(idx.begin(), idx.end(), 0);
    if (ss < n) {
      std::mt19937 rng(42);
      std::shuffle(idx.begin(), idx.end(), rng);
      idx.resize(ss);
    }
    std::vector<float> c(dim, 0.0f);
    for (size_t i : idx)
      for (uint32_t d = 0; d < dim; ++d) c[d] = c[d] + h_vecs[i * dim + d];
    for (uint32_t d = 0; d < dim; ++d) c[d] = c[d] / float(ss);
    float best = std::numeric_limits<float>::max();
    for (size_t i = 0; i < n; ++i) {
      const float d = host_l2_ref(h_vecs + i * dim, c.data(), dim);
      if (d < best) {
        best = d;
        medoid = uint32_t(i);
      }
    }
  }
  // ---- insertion order and random R-regular init (:686-718) ----
  std::vector<uint32_t> order(n);
  {
    std::vector<size_t> o(n);
    std::iota(o.begin(), o.end(), 0);
    std::mt19937 rng(seed);
    std::shuffle(o.begin(), o.end(), rng);
    for (size_t i = 0; i < n; ++i) order[i] = uint32_t(o[i]);
  }
  std::vector<uint32_t> adj(n * R, kEmpty);
  {
    const size_t deg = std::min<size_t>(R, n - 1);
    std::mt19937 init_rng(seed + 1);
    std::uniform_int_distribution<size_t> dist(0, n - 1);
    for (size_t i = 0; i < n; ++i) {
      uint32_t* row = &adj[i * R];
      size_t cnt = 0;
      while (cnt < deg) {
        const size_t j = dist(init_rng);
        if (j == i) continue;
        bool dup = false;
        for (size_t k = 0; k < cnt; ++k)
          if (row[k] == uint32_t(j)) {
            dup = true;
            break;
          }
        if (!dup) row[cnt++] = uint32_t(j);
      }
    }
  }
  // ---- device buffers ----
  std::vector<float> xs(n * vs, 0.f);
  for (size_t i = 0; i < n; ++i) std::memcpy(&xs[i * vs], h_vecs + i * dim, size_t(dim) * 4);
  DevBuf<float> d_x;
  DevBuf<uint32_t> d_adj, d_order, d_new, d_cnt, d_work, d_ovf, d_tg, d_off, d_mem;
  DevBuf<uint64_t> d_seg;
  DVS_CUDA(d_x.alloc(n * vs));
  DVS_CUDA(d_adj.alloc(n * R));
  DVS_CUDA(d_order.alloc(n));
  DVS_CUDA(cudaMemcpy(d_x.p, xs.data(), xs.size() * 4, cudaMemcpyHostToDevice));
  DVS_CUDA(cudaMemcpy(d_adj.p, adj.data(), adj.size() * 4, cudaMemcpyHostToDevice));
  DVS_CUDA(cudaMemcpy(d_order.p, order.data(), n * 4, cudaMemcpyHostToDevice));
  xs.clear();
  xs.shrink_to_fit();

  size_t cap = bp->batch_cap ? bp->batch_cap : std::max<size_t>(1, std::min<size_t>(65536, n * 2 / 100));
  const uint32_t seg_cap = bp->visited_cap ? bp->visited_cap : 16384;
  DVS_CUDA(d_seg.alloc(cap * seg_cap));
  DVS_CUDA(d_cnt.alloc(cap));
  DVS_CUDA(d_new.alloc(cap * R));
  DVS_CUDA(d_work.alloc(4));
  int sms = 0;
  DVS_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, bp->device));
  // search launch shape
  const uint32_t cap_pad = (L + 31) / 32 * 32;
  const uint32_t hcap = std::max(64u, (L * 64 + 31) / 32 * 32);
  const uint32_t wwords = build_warp_words(cap_pad, vs, hcap);
  uint32_t wpb = 1;
  int bps = 0, best = 0;
  for (uint32_t w : {1u, 2u, 4u}) {
    const size_t sm = size_t(w) * wwords * 4;
    if (sm > 227 * 1024) break;
    DVS_CUDA(cudaFuncSetAttribute(build_search_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm)));
    int b = 0;
    DVS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&b, build_search_kernel, int(w * 32), sm));
    if (int(w) * b > best) {
      best = int(w) * b;
      wpb = w;
      bps = b;
    }
  }
  if (best == 0) return fail(DVS_ERR_CAPACITY, "build beam width needs more shared memory than a block has");
  DVS_CUDA(cudaFuncSetAttribute(build_search_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                int(size_t(wpb) * wwords * 4)));
  const uint32_t search_blocks_full = uint32_t(bps) * uint32_t(sms);
  const uint32_t ovf_cap = 1u << 16;
  DVS_CUDA(d_ovf.alloc(size_t(search_blocks_full) * wpb * ovf_cap));
  uint32_t seg_pow2 = 2;
  while (seg_pow2 < seg_cap) seg_pow2 <<= 1;
  const size_t prune_smem = size_t(seg_pow2) * 8;
  if (prune_smem > 227 * 1024) return fail(DVS_ERR_ARG, "visited_cap too large for the shared-memory sort");
  DVS_CUDA(cudaFuncSetAttribute(prune_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(prune_smem)));
  DVS_CUDA(cudaFuncSetAttribute(reverse_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));

  std::vector<uint32_t> new_h(cap * R), cnt_h(cap);
  std::vector<uint32_t> touched_count(n, 0), tg, off, mem;
  uint64_t total_visited = 0;
  size_t pos = 0, bsz = 1, nbatches = 0;
  while (pos < n) {
    const uint32_t nb = uint32_t(std::min(std::min(bsz, cap), n - pos));
    const uint32_t* nodes = d_order.p + pos;
    // (a) search
    BuildSearchArgs sa;
    sa.vecs = d_x.p;
    sa.adj = d_adj.p;
    sa.nodes = nodes;
    sa.seg = d_seg.p;
    sa.seg_count = d_cnt.p;
    sa.work = d_work.p;
    sa.ovf = d_ovf.p;
    sa.vec_stride = vs;
    sa.dim = dim;
    sa.R = R;
    sa.medoid = medoid;
    sa.nb = nb;
    sa.L = L;
    sa.seg_cap = seg_cap;
    sa.hcap = hcap;
    sa.hlimit = hcap / 10 * 8;
    sa.ovf_cap = ovf_cap;
    sa.ovf_limit = ovf_cap / 10 * 8;
    sa.cap_pad = cap_pad;
    DVS_CUDA(cudaMemset(d_work.p, 0, 16));
    const uint32_t blocks = std::max(1u, std::min(search_blocks_full, (nb + wpb - 1) / wpb));
    build_search_kernel<<<blocks, wpb * 32, size_t(wpb) * wwords * 4>>>(sa);
    DVS_CUDA(cudaGetLastError());
    // (b) prune
    PruneArgs pa;
    pa.vecs = d_x.p;
    pa.nodes = nodes;
    pa.seg = d_seg.p;
    pa.seg_count = d_cnt.p;
    pa.new_adj = d_new.p;
    pa.vec_stride = vs;
    pa.dim = dim;
    pa.R = R;
    pa.seg_cap = seg_cap;
    pa.alpha = alpha_build;
    uint32_t work[4];
    DVS_CUDA(cudaMemcpy(work, d_work.p, 16, cudaMemcpyDeviceToHost));
    if (work[1]) {
      cudaEventDestroy(e0);
      cudaEventDestroy(e1);
      return fail(DVS_ERR_CAPACITY, "a build search visited more than " + std::to_string(seg_cap) +
                                        " nodes; raise visited_cap");
    }
    DVS_CUDA(cudaMemcpy(cnt_h.data(), d_cnt.p, size_t(nb) * 4, cudaMemcpyDeviceToHost));
    uint32_t max_cnt = 2;
    for (uint32_t t = 0; t < nb; ++t) max_cnt = std::max(max_cnt, cnt_h[t]);
    uint32_t Pmax = 2;
    while (Pmax < max_cnt) Pmax <<= 1;
    prune_kernel<<<nb, 512, size_t(Pmax) * 8>>>(pa);
    DVS_CUDA(cudaGetLastError());
    // (c) apply
    {
      const uint64_t tot = uint64_t(nb) * R;
      apply_kernel<<<uint32_t((tot + 255) / 256), 256>>>(d_adj.p, nodes, d_new.p, nb, R);
      DVS_CUDA(cudaGetLastError());
    }
    // (d) reverse edges grouped by target, in batch order
    DVS_CUDA(cudaMemcpy(new_h.data(), d_new.p, size_t(nb) * R * 4, cudaMemcpyDeviceToHost));
    for (uint32_t t = 0; t < nb; ++t) total_visited += cnt_h[t];
    tg.clear();
    for (uint32_t t = 0; t < nb; ++t)
      for (uint32_t j = 0; j < R; ++j) {
        const uint32_t v = new_h[size_t(t) * R + j];
        if (v == kEmpty) break;
        if (touched_count[v]++ == 0) tg.push_back(v);
      }
    std::sort(tg.begin(), tg.end());
    off.assign(tg.size() + 1, 0);
    uint32_t max_group = 0;
    for (size_t gi = 0; gi < tg.size(); ++gi) {
      off[gi + 1] = off[gi] + touched_count[tg[gi]];
      max_group = std::max(max_group, touched_count[tg[gi]]);
      touched_count[tg[gi]] = uint32_t(gi);  // reuse as group index
    }
    mem.assign(off.back(), 0);
    {
      std::vector<uint32_t> fill(tg.size(), 0);
      for (uint32_t t = 0; t < nb; ++t)
        for (uint32_t j = 0; j < R; ++j) {
          const uint32_t v = new_h[size_t(t) * R + j];
          if (v == kEmpty) break;
          const uint32_t gi = touched_count[v];
          mem[off[gi] + fill[gi]++] = order[pos + t];
        }
    }
    for (uint32_t v : tg) touched_count[v] = 0;
    if (!tg.empty()) {
      const size_t need = size_t(R + max_group);
      uint32_t P = 2;
      while (P < need) P <<= 1;
      const size_t rsmem = size_t(P) * 8 + size_t(max_group) * 4 + 16;
      if (rsmem > 200 * 1024)
        return fail(DVS_ERR_CAPACITY, "a node received " + std::to_string(max_group) +
                                          " reverse edges in one batch; lower batch_cap");
      DVS_CUDA(d_tg.alloc(tg.size()));
      DVS_CUDA(d_off.alloc(off.size()));
      DVS_CUDA(d_mem.alloc(mem.size()));
      DVS_CUDA(cudaMemcpy(d_tg.p, tg.data(), tg.size() * 4, cudaMemcpyHostToDevice));
      DVS_CUDA(cudaMemcpy(d_off.p, off.data(), off.size() * 4, cudaMemcpyHostToDevice));
      DVS_CUDA(cudaMemcpy(d_mem.p, mem.data(), mem.size() * 4, cudaMemcpyHostToDevice));
      ReverseArgs ra;
      ra.vecs = d_x.p;
      ra.adj = d_adj.p;
      ra.targets = d_tg.p;
      ra.offsets = d_off.p;
      ra.members = d_mem.p;
      ra.vec_stride = vs;
      ra.dim = dim;
      ra.R = R;
      ra.key_cap = P;
      ra.alpha = alpha_build;
      reverse_kernel<<<uint32_t(tg.size()), 256, rsmem>>>(ra);
      DVS_CUDA(cudaGetLastError());
      DVS_CUDA(cudaDeviceSynchronize());
    }
    pos += nb;
    bsz = std::min(bsz * 2, cap);
    ++nbatches;
  }
  DVS_CUDA(cudaMemcpy(adj.data(), d_adj.p, adj.size() * 4, cudaMemcpyDeviceToHost));
  DVS_CUDA(cudaEventRecord(e1));
  DVS_CUDA(cudaEventSynchronize(e1));
  float graph_ms = 0.f;
  DVS_CUDA(cudaEventElapsedTime(&graph_ms, e0, e1));

  // ---- RaBitQ artifacts (init_rabitq :978-1024) and records ----
  std::vector<float> P;
  rotation_matrix(dim, int(bp->seed), P);
  std::vector<float> cen(dim, 0.0f), c_rot(dim, 0.0f);
  for (size_t i = 0; i < n; ++i)
    for (uint32_t d = 0; d < dim; ++d) cen[d] = cen[d] + h_vecs[i * dim + d];
  for (uint32_t d = 0; d < dim; ++d) cen[d] = cen[d] / float(n);
  for (uint32_t j = 0; j < dim; ++j) {
    float acc = 0.f;
    for (uint32_t i = 0; i < dim; ++i) acc = std::fmaf(P[size_t(j) * dim + i], cen[i], acc);
    c_rot[j] = acc;
  }
  const double tc = dvs::t_const(dim, bits, uint64_t(int64_t(bp->seed)));
  const uint32_t rs = (bits * dim + 7) / 8 + 8;
  std::vector<uint8_t> rec(size_t(n) * rs);
  {
    DevBuf<float> d_P, d_c;
    DevBuf<uint8_t> d_rec;
    DVS_CUDA(d_P.alloc(size_t(dim) * dim));
    DVS_CUDA(d_c.alloc(dim));
    DVS_CUDA(d_rec.alloc(rec.size()));
    DVS_CUDA(cudaMemcpy(d_P.p, P.data(), P.size() * 4, cudaMemcpyHostToDevice));
    DVS_CUDA(cudaMemcpy(d_c.p, c_rot.data(), dim * 4, cudaMemcpyHostToDevice));
    const uint32_t grid = uint32_t(std::min<uint64_t>(n, uint64_t(sms) * 16));
    quantize_kernel<<<grid, 128, size_t(dim) * 8 + dim + 16>>>(d_x.p, vs, d_P.p, d_c.p, tc, dim, bits, uint32_t(n),
                                                                d_rec.p, rs);
    DVS_CUDA(cudaGetLastError());
    DVS_CUDA(cudaMemcpy(rec.data(), d_rec.p, rec.size(), cudaMemcpyDeviceToHost));
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (stats) {
    stats->medoid = medoid;
    stats->batches = nbatches;
    stats->graph_ms = graph_ms;
    stats->mean_visited = double(total_visited) / double(n);
    uint64_t edges = 0;
    for (uint32_t v : adj) edges += v != kEmpty;
    stats->mean_degree = double(edges) / double(n);
  }
  if (bp->out_adj) std::memcpy(bp->out_adj, adj.data(), adj.size() * 4);
  if (bp->out_records) std::memcpy(bp->out_records, rec.data(), rec.size());
  if (!bp->output_prefix) return DVS_OK;
  dvs_write_params wp{};
  wp.index_prefix = bp->output_prefix;
  wp.num_vectors = n;
  wp.dim = dim;
  wp.R = R;
  wp.rabitq_bits = bits;
  wp.num_memory_nodes = bp->num_memory_nodes ? bp->num_memory_nodes : 1;
  wp.medoid = medoid;
  wp.beam_width = L;
  wp.alpha = bp->alpha;
  wp.metric = bp->metric;
  wp.t_const = tc;
  return dvs_write_index(&wp, h_vecs, adj.data(), rec.data(), P.data(), c_rot.data(), nullptr);
}

}  // extern "C"
