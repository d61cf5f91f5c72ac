// Online insert into a device-resident index: Vamana::insert
// (src/vamana/vamana.hh:458-999) for batches of vectors.
//
// The reference inserts one vector per coroutine: an exact-distance beam
// search of capacity L_c over RDMA, a sort of the final beam, GPU RobustPrune
// (robust_prune_kernel), GPU quantization (rabitq_quantize_single_kernel), a
// node write, then one locked read-modify-write per selected neighbour (append
// when the list has room, else RobustPrune of the neighbour's list plus the new
// node).  Here a step of b vectors runs as five launches on the device that
// holds the index:
//   1. search_kernel in exact mode (capacity L_c), the final beam as dense slots;
//   2. rotation (the query-prepare kernels) + insert_quantize_kernel (the float
//      GPU quantizer, one lane quad per vector, the reference's 4-lane split);
//   3. insert_prune_kernel (one block per vector) writes the new adjacency rows;
//   4. vectors and ids are appended;
//   5. reverse_edges_kernel: one warp per old node that gains an edge, applying
//      its incoming new nodes in insert order (append, or RobustPrune of its
//      R neighbours + the new node by batch_l2_squared_distance_kernel order).
// Every vector of a step searches the graph as it stood when the step began;
// with steps of one vector this is the reference's sequential insert.  Steps
// never hold more vectors than the index has nodes, and an empty index first
// takes one vector as its medoid (vamana.hh:479-546).

#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <vector>

#include <cub/cub.cuh>
#include <cuda_pipeline.h>

#include "device_math.cuh"
#include "index_state.h"

using dvs::fail;

namespace dvs {
namespace {

// |a - b|^2 as one sequential fma chain over dims 0..dim-1 (the order of
// robust_prune_kernel's `dist += diff * diff`).  Rows are 16-byte aligned;
// 32 dims are loaded per batch so a distance waits on memory dim/32 times.
__device__ __forceinline__ float chain_l2(const float* __restrict__ a, const float* __restrict__ b, uint32_t dim) {
  const float4* a4 = reinterpret_cast<const float4*>(a);
  const float4* b4 = reinterpret_cast<const float4*>(b);
  const uint32_t n4 = dim >> 2;
  float d = 0.f;
  uint32_t k4 = 0;
  for (; k4 + 8 <= n4; k4 += 8) {
    float4 x[8], y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      x[j] = a4[k4 + j];
      y[j] = b4[k4 + j];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float t = __fsub_rn(x[j].x, y[j].x);
      d = __fmaf_rn(t, t, d);
      t = __fsub_rn(x[j].y, y[j].y);
      d = __fmaf_rn(t, t, d);
      t = __fsub_rn(x[j].z, y[j].z);
      d = __fmaf_rn(t, t, d);
      t = __fsub_rn(x[j].w, y[j].w);
      d = __fmaf_rn(t, t, d);
    }
  }
  for (uint32_t k = k4 * 4; k < dim; ++k) {
    const float t = __fsub_rn(a[k], b[k]);
    d = __fmaf_rn(t, t, d);
  }
  return d;
}

constexpr uint32_t kQuantPerBlock = 8;    // vectors per quantize block (one lane quad each)
constexpr uint32_t kPruneThreads = 128;
constexpr uint32_t kRevWarps = 4;         // warps (targets in flight) per reverse-edge block
constexpr uint32_t kMaxAll = 65;          // R + 1 candidates of an overflow prune (R <= 64)
constexpr size_t kStageBudget = 160 * 1024;  // shared memory for staged candidate vectors per block
// largest reverse-edge warp that stages its candidate rows; wider rows go to
// the block-per-target kernel, which shares one staging among four warps
constexpr size_t kRevStageMax = 32 * 1024;

// rabitq_quantize_single_kernel<4,B> (src/gpu/kernels/distance_kernels.cuh:376-464)
// on rotated rows: lane t of a quad takes dims j = t mod 4; tile sums by the
// butterfly; IEEE division and square root; the double t_const*|o| + 1e-5 as
// one double fma, every `acc += a*b` as an fma (nvcc's contractions).  Writes
// the record in the device layout at row row0 + v.
__global__ void __launch_bounds__(32) insert_quantize_kernel(const float* __restrict__ qrot, uint32_t qstride,
                                                              const float* __restrict__ c, double tc, uint32_t dim,
                                                              uint32_t bits, uint32_t nvec, uint32_t* __restrict__ rec,
                                                              uint32_t rec_words, uint32_t code_words, uint64_t row0) {
  extern __shared__ uint8_t u_all[];
  const uint32_t lane = threadIdx.x & 31, t = lane & 3, qd = lane >> 2;
  const uint32_t v = blockIdx.x * kQuantPerBlock + qd;
  const bool live = v < nvec;
  uint8_t* u = u_all + size_t(qd) * dim;
  const float* r = qrot + size_t(live ? v : 0) * qstride;
  float l2p = 0.f;
  if (live)
    for (uint32_t j = t; j < dim; j += 4) {
      const float diff = __fsub_rn(r[j], c[j]);
      l2p = __fmaf_rn(diff, diff, l2p);
    }
  const float l2_sqr = quad_butterfly(l2p);
  const float l2_norm = __fsqrt_rn(l2_sqr);
  const int top = 1 << (bits - 1);
  float ipp = 0.f;
  if (live)
    for (uint32_t j = t; j < dim; j += 4) {
      const float abs_o = fabsf(__fdiv_rn(__fsub_rn(r[j], c[j]), l2_norm));
      int val = static_cast<int>(__fma_rn(tc, static_cast<double>(abs_o), 1e-5));
      if (val >= top) val = top - 1;
      u[j] = static_cast<uint8_t>(val);
      ipp = __fmaf_rn(__fadd_rn(static_cast<float>(val), 0.5f), abs_o, ipp);
    }
  const float ip_norm = quad_butterfly(ipp);
  const float ip_norm_inv = ip_norm == 0.f ? 1.f : __fdiv_rn(1.f, ip_norm);
  const uint32_t mask = uint32_t(top) - 1u;
  if (live)
    for (uint32_t j = t; j < dim; j += 4) {
      if (__fsub_rn(r[j], c[j]) >= 0.f)
        u[j] = static_cast<uint8_t>(u[j] + top);
      else
        u[j] = static_cast<uint8_t>((~u[j]) & mask);
    }
  const float cb = -__fsub_rn(static_cast<float>(top), 0.5f);
  float rx = 0.f, cx = 0.f;
  if (live)
    for (uint32_t j = t; j < dim; j += 4) {
      const float residual = __fsub_rn(r[j], c[j]);
      const float xu_cb = __fadd_rn(static_cast<float>(u[j]), cb);
      rx = __fmaf_rn(residual, xu_cb, rx);
      cx = __fmaf_rn(c[j], xu_cb, cx);
    }
  float ip_resi = quad_butterfly(rx);
  const float ip_cent = quad_butterfly(cx);
  if (ip_resi == 0.f) ip_resi = FLT_MAX;
  const float add = __fadd_rn(l2_sqr, __fdiv_rn(__fmul_rn(__fmul_rn(2.f, l2_sqr), ip_cent), ip_resi));
  const float rescale = __fmul_rn(__fmul_rn(ip_norm_inv, -2.f), l2_norm);
  __syncwarp();
  if (!live) return;
  uint32_t* rr = rec + (row0 + v) * rec_words;
  const uint32_t packed = (bits * dim + 7) / 8, per = 8 / bits;
  for (uint32_t w = t; w < rec_words; w += 4) {
    uint32_t word = 0;
    if (w < code_words) {
      for (uint32_t k = 0; k < 4; ++k) {
        const uint32_t b = 4 * w + k;
        if (b >= packed) break;
        uint32_t byte = 0;
        for (uint32_t e = 0; e < per && b * per + e < dim; ++e) byte |= uint32_t(u[b * per + e]) << (e * bits);
        word |= byte << (8 * k);
      }
    } else if (w == code_words) {
      word = __float_as_uint(add);
    } else if (w == code_words + 1) {
      word = __float_as_uint(rescale);
    }
    rr[w] = word;
  }
}

// float4s between the starts of two staged candidate rows of a prune:
// vec_stride / 4 rounded up to odd, so threads reading consecutive rows at one
// offset fall in distinct banks.
__host__ __device__ inline uint32_t prune_row_stride4(uint32_t vec_stride) { return (vec_stride >> 2) | 1u; }

// robust_prune_kernel (src/gpu/kernels/distance_kernels.cuh:285-370) for new
// vector v: its final beam (slots by ascending distance, from the search) is
// the candidate list; the nearest valid candidate is kept and every later
// valid p' with alpha * |p* - p'|^2 <= d(v, p') is dropped, until R are kept.
// The kept slots are the new node's adjacency row (row0 + v).  The
// candidates' vectors are copied to shared memory once (cp.async) at an odd
// float4 stride, so the greedy loop reads no global memory and threads reading
// consecutive candidates hit distinct banks.  Used when Lc rows fit; wider
// rows go to insert_prune_passes_kernel.
__global__ void __launch_bounds__(kPruneThreads) insert_prune_kernel(const DevLayout ix, const uint32_t* __restrict__ cand,
                                                                     const float* __restrict__ cand_d,
                                                                     const uint32_t* __restrict__ counters, uint32_t Lc,
                                                                     float alpha, uint64_t row0,
                                                                     uint32_t* __restrict__ adj) {
  extern __shared__ __align__(16) float sm[];
  const uint32_t v = blockIdx.x, tid = threadIdx.x, R = ix.R, dim = ix.dim, vs = ix.vec_stride;
  const uint32_t rs = 4 * prune_row_stride4(vs);  // floats between staged rows
  float* rows = sm;                               // Lc candidate vectors
  float* dd = rows + size_t(Lc) * rs;             // candidate distances
  uint32_t* sl = reinterpret_cast<uint32_t*>(dd + Lc);  // candidate slots
  uint8_t* valid = reinterpret_cast<uint8_t*>(sl + Lc);
  const uint32_t n = counters[size_t(v) * 4 + 3] & 0xFFFFu;
  for (uint32_t i = tid; i < n; i += blockDim.x) {
    dd[i] = cand_d[size_t(v) * Lc + i];
    sl[i] = cand[size_t(v) * Lc + i];
    valid[i] = 1;
  }
  __syncthreads();
  uint32_t* row = adj + (row0 + v) * R;
  if (n <= R) {
    for (uint32_t j = tid; j < R; j += blockDim.x) row[j] = j < n ? sl[j] : kEmptySlot;
    return;
  }
  const uint32_t c4 = vs >> 2;
  for (uint32_t idx = tid; idx < n * c4; idx += blockDim.x) {
    const uint32_t r = idx / c4, c = idx - r * c4;
    __pipeline_memcpy_async(reinterpret_cast<float4*>(rows + size_t(r) * rs) + c,
                            reinterpret_cast<const float4*>(vec_row(ix, sl[r])) + c, 16);
  }
  __pipeline_commit();
  __pipeline_wait_prior(0);
  __syncthreads();
  uint32_t kept = 0;  // identical in every thread
  for (uint32_t s = 0; s < n && kept < R; ++s) {
    if (!valid[s]) continue;
    if (tid == 0) row[kept] = sl[s];
    ++kept;
    const float* pv = rows + size_t(s) * rs;
    for (uint32_t i = s + 1 + tid; i < n; i += blockDim.x) {
      if (!valid[i]) continue;
      const float d = chain_l2(pv, rows + size_t(i) * rs, dim);
      if (__fmul_rn(alpha, d) <= dd[i]) valid[i] = 0;
    }
    __syncthreads();
  }
  for (uint32_t j = kept + tid; j < R; j += blockDim.x) row[j] = kEmptySlot;
}

constexpr uint32_t kPivots = 8;  // pivot candidates per pass of insert_prune_passes_kernel

// |p_k - x|^2 for the np <= kPivots pivot rows p_k (shared memory, stride vs
// floats) against one candidate row x (global): np fma chains over dims
// 0..dim-1 in order (each the chain of chain_l2, pivot minus candidate), the
// candidate's chunks read once for all of them.
__device__ __forceinline__ void chain_l2_pivots(const float* prow, uint32_t vs, uint32_t np, const float* x,
                                                uint32_t dim, float (&out)[kPivots]) {
  const float4* x4 = reinterpret_cast<const float4*>(x);
  const uint32_t n4 = dim >> 2, s4 = vs >> 2;
  const float4* p4 = reinterpret_cast<const float4*>(prow);
  float d[kPivots];
#pragma unroll
  for (int p = 0; p < int(kPivots); ++p) d[p] = 0.f;
#define DVS_CHP(Y, X, D)                                   \
  {                                                        \
    float t = __fsub_rn(Y.x, X.x); D = __fmaf_rn(t, t, D); \
    t = __fsub_rn(Y.y, X.y); D = __fmaf_rn(t, t, D);       \
    t = __fsub_rn(Y.z, X.z); D = __fmaf_rn(t, t, D);       \
    t = __fsub_rn(Y.w, X.w); D = __fmaf_rn(t, t, D);       \
  }
  uint32_t k4 = 0;
  for (; k4 + 4 <= n4; k4 += 4) {
    float4 a[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) a[c] = __ldg(x4 + k4 + c);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
      for (int p = 0; p < int(kPivots); ++p)
        if (uint32_t(p) < np) {
          const float4 y = p4[size_t(p) * s4 + k4 + c];
          DVS_CHP(y, a[c], d[p])
        }
    }
  }
  for (; k4 < n4; ++k4) {
    const float4 a = __ldg(x4 + k4);
#pragma unroll
    for (int p = 0; p < int(kPivots); ++p)
      if (uint32_t(p) < np) {
        const float4 y = p4[size_t(p) * s4 + k4];
        DVS_CHP(y, a, d[p])
      }
  }
#undef DVS_CHP
  for (uint32_t k = n4 * 4; k < dim; ++k) {
    const float xv = __ldg(x + k);
#pragma unroll
    for (int p = 0; p < int(kPivots); ++p)
      if (uint32_t(p) < np) {
        const float t = __fsub_rn(prow[size_t(p) * vs + k], xv);
        d[p] = __fmaf_rn(t, t, d[p]);
      }
  }
#pragma unroll
  for (int p = 0; p < int(kPivots); ++p) out[p] = d[p];
}

// Shared memory of insert_prune_passes_kernel: kPivots pivot rows, kPivots x Lc
// pivot distances, candidate distances and slots, pass words, valid flags.
inline size_t prune_passes_bytes(uint32_t Lc, uint32_t vec_stride) {
  return size_t(kPivots) * vec_stride * 4 + size_t(kPivots) * Lc * 4 + size_t(Lc) * 8 + (kPivots + 4) * 4 + Lc + 16;
}

// insert_prune_kernel for rows too wide to stage all Lc candidates: the greedy
// pass in passes of up to kPivots pivots.  A pass takes the next kPivots valid
// candidates (in rank order) as the pivots it may keep, stages their rows, and
// reads each later valid candidate's row once for the distances to all of them;
// warp 0 then walks those pivots in rank order, keeping each one still valid
// and dropping the later candidates it prunes.  A rank skipped between two
// pivots was invalid before the pass began, so the kept list is the one the
// step-by-step pass gives, from the same chains, with a pass per kPivots kept
// (or pruned) pivots instead of a read of every candidate row per kept one.
__global__ void __launch_bounds__(kPruneThreads) insert_prune_passes_kernel(
    const DevLayout ix, const uint32_t* __restrict__ cand, const float* __restrict__ cand_d,
    const uint32_t* __restrict__ counters, uint32_t Lc, float alpha, uint64_t row0, uint32_t* __restrict__ adj) {
  extern __shared__ __align__(16) float sm[];
  const uint32_t v = blockIdx.x, tid = threadIdx.x, lane = tid & 31, R = ix.R, dim = ix.dim, vs = ix.vec_stride;
  const uint32_t c4 = vs >> 2;
  float* prow = sm;                                        // kPivots pivot rows
  float* dp = prow + size_t(kPivots) * vs;                 // dp[p * Lc + i] = |pivot p - candidate i|^2
  float* dd = dp + size_t(kPivots) * Lc;                   // candidate distances
  uint32_t* sl = reinterpret_cast<uint32_t*>(dd + Lc);     // candidate slots
  uint32_t* piv = sl + Lc;                                 // pivot ranks, [kPivots] count, [kPivots + 1] kept
  uint8_t* valid = reinterpret_cast<uint8_t*>(piv + kPivots + 4);
  const uint32_t n = counters[size_t(v) * 4 + 3] & 0xFFFFu;
  for (uint32_t i = tid; i < n; i += blockDim.x) {
    dd[i] = cand_d[size_t(v) * Lc + i];
    sl[i] = cand[size_t(v) * Lc + i];
    valid[i] = 1;
  }
  __syncthreads();
  uint32_t* row = adj + (row0 + v) * R;
  if (n <= R) {
    for (uint32_t j = tid; j < R; j += blockDim.x) row[j] = j < n ? sl[j] : kEmptySlot;
    return;
  }
  uint32_t kept = 0, cur = 0;  // identical in every thread
  while (kept < R) {
    if (tid < 32) {
      uint32_t np = 0;
      for (uint32_t b = cur; b < n && np < kPivots; b += 32) {
        uint32_t msk = __ballot_sync(0xFFFFFFFFu, b + lane < n && valid[b + lane]);
        while (msk && np < kPivots) {
          if (lane == 0) piv[np] = b + __ffs(msk) - 1;
          ++np;
          msk &= msk - 1;
        }
      }
      if (lane == 0) piv[kPivots] = np;
    }
    __syncthreads();
    const uint32_t np = piv[kPivots];
    if (np == 0) break;
    for (uint32_t idx = tid; idx < np * c4; idx += blockDim.x) {
      const uint32_t p = idx / c4, c = idx - p * c4;
      __pipeline_memcpy_async(reinterpret_cast<float4*>(prow + size_t(p) * vs) + c,
                              reinterpret_cast<const float4*>(vec_row(ix, sl[piv[p]])) + c, 16);
    }
    __pipeline_commit();
    __pipeline_wait_prior(0);
    __syncthreads();
    for (uint32_t i = piv[0] + 1 + tid; i < n; i += blockDim.x) {
      if (!valid[i]) continue;
      float out[kPivots];
      chain_l2_pivots(prow, vs, np, vec_row(ix, sl[i]), dim, out);
#pragma unroll
      for (int p = 0; p < int(kPivots); ++p)
        if (uint32_t(p) < np) dp[size_t(p) * Lc + i] = out[p];
    }
    __syncthreads();
    if (tid < 32) {
      uint32_t k2 = kept;
      for (uint32_t p = 0; p < np && k2 < R; ++p) {
        const uint32_t s = piv[p];
        if (!valid[s]) continue;
        if (lane == 0) row[k2] = sl[s];
        ++k2;
        for (uint32_t i = s + 1 + lane; i < n; i += 32)
          if (valid[i] && __fmul_rn(alpha, dp[size_t(p) * Lc + i]) <= dd[i]) valid[i] = 0;
        __syncwarp();
      }
      if (lane == 0) piv[kPivots + 1] = k2;
    }
    __syncthreads();
    kept = piv[kPivots + 1];
    cur = piv[np - 1] + 1;
    __syncthreads();  // every thread has read the pass words before the next pass rewrites them
  }
  for (uint32_t j = kept + tid; j < R; j += blockDim.x) row[j] = kEmptySlot;
}

struct RevWarp {
  uint32_t all[kMaxAll];
  uint32_t order[kMaxAll];
  float d[kMaxAll];
  float sd[kMaxAll];
  uint32_t kept[64];
  uint8_t valid[kMaxAll + 3];
};
constexpr size_t kRevWarpBytes = (sizeof(RevWarp) + 15) / 16 * 16;

// Shared memory of one reverse-edge warp: its RevWarp, then (STAGED) the R + 1
// candidate rows.
__host__ __device__ inline size_t rev_warp_bytes(uint32_t R, uint32_t vec_stride, bool staged) {
  return kRevWarpBytes + (staged ? size_t(R + 1) * prune_row_stride4(vec_stride) * 16 : 0);
}

// Reverse edges (vamana.hh:795-986): warp w takes old node targets[w] and
// applies the new slots srcs[offs[w] .. offs[w+1]) in insert order (*nruns
// groups; a group keyed by the empty slot is skipped).  A list with room gets
// the new slot appended; a full one is replaced by RobustPrune of its R
// neighbours plus the new node, from the target's vector, with the distances
// of batch_l2_squared_distance_kernel<4> ordered by (distance, position).
// The candidates' vectors are read from global memory for those distances
// (two per lane quad); STAGED then copies them to shared memory in rank order
// (cp.async), so that in the greedy loop lane l reads rank s + 1 + l, rows at
// an odd float4 stride: no bank conflicts, the pivot row a broadcast.
// stats[2] counts the overflow prunes, stats[3] keeps the largest group.
template <bool STAGED>
__global__ void __launch_bounds__(kRevWarps * 32) reverse_edges_kernel(const DevLayout ix, uint32_t* __restrict__ adj,
                                                                       const uint32_t* __restrict__ targets,
                                                                       const uint32_t* __restrict__ offs,
                                                                       const uint32_t* __restrict__ srcs,
                                                                       const uint32_t* __restrict__ nruns, float alpha,
                                                                       unsigned long long* __restrict__ stats) {
  extern __shared__ __align__(16) uint8_t rev_smem[];
  const uint32_t lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const uint32_t R = ix.R, dim = ix.dim, c4 = ix.vec_stride >> 2, s4 = prune_row_stride4(ix.vec_stride);
  uint8_t* mine = rev_smem + size_t(wib) * rev_warp_bytes(R, ix.vec_stride, STAGED);
  RevWarp& W = *reinterpret_cast<RevWarp*>(mine);
  float4* rows = reinterpret_cast<float4*>(mine + kRevWarpBytes);
  const uint32_t wpb = blockDim.x >> 5;
  const uint32_t ntargets = *nruns;
  for (uint32_t w = blockIdx.x * wpb + wib; w < ntargets; w += gridDim.x * wpb) {
    const uint32_t tg = targets[w];
    if (tg == kEmptySlot) continue;
    uint32_t* row = adj + size_t(tg) * R;
    if (lane == 0) atomicMax(stats + 3, static_cast<unsigned long long>(offs[w + 1] - offs[w]));
    const float* tv = vec_row(ix, tg);
    for (uint32_t e = offs[w]; e < offs[w + 1]; ++e) {
      const uint32_t v = srcs[e];
      const uint32_t a0 = lane < R ? row[lane] : kEmptySlot;
      const uint32_t a1 = lane + 32 < R ? row[lane + 32] : kEmptySlot;
      const uint32_t cnt = __popc(__ballot_sync(0xFFFFFFFFu, a0 != kEmptySlot)) +
                           __popc(__ballot_sync(0xFFFFFFFFu, a1 != kEmptySlot));
      __syncwarp();
      if (cnt < R) {
        if (lane == 0) row[cnt] = v;
        __syncwarp();
        continue;
      }
      if (lane == 0) atomicAdd(stats + 2, 1ull);
      const uint32_t n_all = R + 1;
      if (lane < R) W.all[lane] = a0;
      if (lane + 32 < R) W.all[lane + 32] = a1;
      if (lane == 0) W.all[R] = v;
      __syncwarp();
      for (uint32_t i0 = 0; i0 < n_all; i0 += 16) {
        const uint32_t iA = i0 + (lane >> 2), iB = iA + 8;
        float pA = 0.f, pB = 0.f;
        if (iA < n_all) {
          const float* xA = vec_row(ix, W.all[iA]);
          const float* xB = iB < n_all ? vec_row(ix, W.all[iB]) : xA;
          l2_quad_partial2(tv, xA, xB, dim, lane & 3, pA, pB);
        }
        const float tA = quad_butterfly(pA), tB = quad_butterfly(pB);
        if ((lane & 3) == 0) {
          if (iA < n_all) W.d[iA] = tA;
          if (iB < n_all) W.d[iB] = tB;
        }
      }
      __syncwarp();
      for (uint32_t i = lane; i < n_all; i += 32) {
        const float di = W.d[i];
        uint32_t rk = 0;
        for (uint32_t j = 0; j < n_all; ++j) rk += (W.d[j] < di) || (W.d[j] == di && j < i);
        W.order[rk] = i;
        W.sd[rk] = di;
        W.valid[rk] = 1;
      }
      __syncwarp();
      if (STAGED) {
        for (uint32_t idx = lane; idx < n_all * c4; idx += 32) {
          const uint32_t r = idx / c4, c = idx - r * c4;
          __pipeline_memcpy_async(rows + size_t(r) * s4 + c,
                                  reinterpret_cast<const float4*>(vec_row(ix, W.all[W.order[r]])) + c, 16);
        }
        __pipeline_commit();
        __pipeline_wait_prior(0);
        __syncwarp();
      }
      auto ranked_row = [&](uint32_t s) -> const float* {
        return STAGED ? reinterpret_cast<const float*>(rows + size_t(s) * s4) : vec_row(ix, W.all[W.order[s]]);
      };
      uint32_t kept = 0;
      for (uint32_t s = 0; s < n_all && kept < R; ++s) {
        if (!W.valid[s]) continue;
        if (lane == 0) W.kept[kept] = W.all[W.order[s]];
        ++kept;
        const float* pv = ranked_row(s);
        for (uint32_t i = s + 1 + lane; i < n_all; i += 32) {
          if (!W.valid[i]) continue;
          const float d = chain_l2(pv, ranked_row(i), dim);
          if (__fmul_rn(alpha, d) <= W.sd[i]) W.valid[i] = 0;
        }
        __syncwarp();
      }
      for (uint32_t j = lane; j < R; j += 32) row[j] = j < kept ? W.kept[j] : kEmptySlot;
      __syncwarp();
    }
  }
}

// l2_quad_partial2's two chains (float4 chunks t, t+4, ... then tail dim
// n4*4 + t, diff = q - x) with plain loads, so the rows may be in shared memory.
__device__ __forceinline__ void l2_quad2_any(const float* q, const float* xA, const float* xB, uint32_t dim,
                                             uint32_t t, float& accA, float& accB) {
  const uint32_t n4 = dim >> 2;
  const float4* q4 = reinterpret_cast<const float4*>(q);
  const float4* a4 = reinterpret_cast<const float4*>(xA);
  const float4* b4 = reinterpret_cast<const float4*>(xB);
  float sa = 0.f, sb = 0.f;
  for (uint32_t i = t; i < n4; i += 4) {
    const float4 c = q4[i], a = a4[i], b = b4[i];
    float d;
    d = __fsub_rn(c.x, a.x); sa = __fmaf_rn(d, d, sa);
    d = __fsub_rn(c.x, b.x); sb = __fmaf_rn(d, d, sb);
    d = __fsub_rn(c.y, a.y); sa = __fmaf_rn(d, d, sa);
    d = __fsub_rn(c.y, b.y); sb = __fmaf_rn(d, d, sb);
    d = __fsub_rn(c.z, a.z); sa = __fmaf_rn(d, d, sa);
    d = __fsub_rn(c.z, b.z); sb = __fmaf_rn(d, d, sb);
    d = __fsub_rn(c.w, a.w); sa = __fmaf_rn(d, d, sa);
    d = __fsub_rn(c.w, b.w); sb = __fmaf_rn(d, d, sb);
  }
  const uint32_t tail = (n4 << 2) + t;
  if (tail < dim) {
    float d = __fsub_rn(q[tail], xA[tail]);
    sa = __fmaf_rn(d, d, sa);
    d = __fsub_rn(q[tail], xB[tail]);
    sb = __fmaf_rn(d, d, sb);
  }
  accA = sa;
  accB = sb;
}

// d(a, b_k), k < P, as P fma chains over dims 0..dim-1 in order (each the
// chain of chain_l2), interleaved; four chunks of every row per batch.
// Rows are 16-byte aligned, in shared or global memory.
template <int P>
__device__ __forceinline__ void chain_l2_multi(const float* a, const float* const (&b)[P], uint32_t dim,
                                               float (&out)[P]) {
  const float4* a4 = reinterpret_cast<const float4*>(a);
  const float4* bs[P];
#pragma unroll
  for (int r = 0; r < P; ++r) bs[r] = reinterpret_cast<const float4*>(b[r]);
  float d[P];
#pragma unroll
  for (int r = 0; r < P; ++r) d[r] = 0.f;
  const uint32_t n4 = dim >> 2;
  uint32_t k4 = 0;
#define DVS_CH4(X, Y, D)                                   \
  {                                                        \
    float t = __fsub_rn(X.x, Y.x); D = __fmaf_rn(t, t, D); \
    t = __fsub_rn(X.y, Y.y); D = __fmaf_rn(t, t, D);       \
    t = __fsub_rn(X.z, Y.z); D = __fmaf_rn(t, t, D);       \
    t = __fsub_rn(X.w, Y.w); D = __fmaf_rn(t, t, D);       \
  }
  for (; k4 + 4 <= n4; k4 += 4) {
    float4 x[4], y[P][4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      x[c] = a4[k4 + c];
#pragma unroll
      for (int r = 0; r < P; ++r) y[r][c] = bs[r][k4 + c];
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
      for (int r = 0; r < P; ++r) DVS_CH4(x[c], y[r][c], d[r])
    }
  }
  for (; k4 < n4; ++k4) {
    const float4 x = a4[k4];
#pragma unroll
    for (int r = 0; r < P; ++r) {
      const float4 y = bs[r][k4];
      DVS_CH4(x, y, d[r])
    }
  }
#undef DVS_CH4
  for (uint32_t k = n4 * 4; k < dim; ++k) {
#pragma unroll
    for (int r = 0; r < P; ++r) {
      const float t = __fsub_rn(a[k], b[r][k]);
      d[r] = __fmaf_rn(t, t, d[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < P; ++r) out[r] = d[r];
}

constexpr uint32_t kRevThreads = 256;  // threads of a reverse-edge block (one target node at a time)
constexpr uint32_t kRevPartners = 4;   // pair distances per item (chains a thread runs at once)

// Pair items of row i of n candidates: its n - 1 - i later partners,
// kRevPartners per item.
__host__ __device__ inline uint32_t row_items(uint32_t n, uint32_t i) {
  return (n - 1 - i + kRevPartners - 1) / kRevPartners;
}
__host__ __device__ inline uint32_t item_count(uint32_t n) {
  uint32_t t = 0;
  for (uint32_t i = 0; i < n; ++i) t += row_items(n, i);
  return t;
}

// Shared memory of a reverse-edge block: its RevWarp, the (R+1)^2 pair
// distances, the R + 1 candidate rows (index order, odd float4 stride).
__host__ __device__ inline size_t rev_pairs_bytes(uint32_t R) { return (size_t(R + 1) * (R + 1) * 4 + 15) / 16 * 16; }
__host__ __device__ inline size_t rev_block_bytes(uint32_t R, uint32_t vec_stride) {
  return kRevWarpBytes + rev_pairs_bytes(R) + size_t(R + 1) * prune_row_stride4(vec_stride) * 16;
}

// reverse_edges_kernel for wide rows, where a warp's staged rows would leave
// few warps per SM: a block of kRevThreads per target shares one staging of
// the R + 1 candidate rows (cp.async), computes the distances to the target
// from there, and then every pair distance of the candidates up front, four
// chains per thread at once (thread m of row i's items takes partners
// i+1+m + Q*q, q < kRevPartners, Q = row i's item count, so neighbouring threads read
// neighbouring rows: no bank conflicts).  Warp 0 then runs the greedy pass on
// those values.  Each value is the chain the step-by-step pass computes for
// that pair (|a-b|^2 is the same chain either way round: a-b and b-a differ
// only in sign), so the kept list is the same.
__global__ void __launch_bounds__(kRevThreads) reverse_edges_block_kernel(const DevLayout ix, uint32_t* __restrict__ adj,
                                                                         const uint32_t* __restrict__ targets,
                                                                         const uint32_t* __restrict__ offs,
                                                                         const uint32_t* __restrict__ srcs,
                                                                         const uint32_t* __restrict__ nruns,
                                                                         float alpha,
                                                                         unsigned long long* __restrict__ stats) {
  extern __shared__ __align__(16) uint8_t rev_smem[];
  const uint32_t tid = threadIdx.x, lane = tid & 31;
  const uint32_t R = ix.R, dim = ix.dim, c4 = ix.vec_stride >> 2, s4 = prune_row_stride4(ix.vec_stride);
  const uint32_t n = R + 1;
  RevWarp& B = *reinterpret_cast<RevWarp*>(rev_smem);
  float* Dm = reinterpret_cast<float*>(rev_smem + kRevWarpBytes);
  float4* rows = reinterpret_cast<float4*>(rev_smem + kRevWarpBytes + rev_pairs_bytes(R));
  __shared__ uint32_t cnt_s;
  const uint32_t ntargets = *nruns;
  for (uint32_t w = blockIdx.x; w < ntargets; w += gridDim.x) {
    const uint32_t tg = targets[w];
    if (tg == kEmptySlot) continue;
    uint32_t* row = adj + size_t(tg) * R;
    if (tid == 0) atomicMax(stats + 3, static_cast<unsigned long long>(offs[w + 1] - offs[w]));
    const float* tv = vec_row(ix, tg);
    for (uint32_t e = offs[w]; e < offs[w + 1]; ++e) {
      const uint32_t v = srcs[e];
      if (tid < 32) {
        const uint32_t a0 = lane < R ? row[lane] : kEmptySlot;
        const uint32_t a1 = lane + 32 < R ? row[lane + 32] : kEmptySlot;
        const uint32_t cnt = __popc(__ballot_sync(0xFFFFFFFFu, a0 != kEmptySlot)) +
                             __popc(__ballot_sync(0xFFFFFFFFu, a1 != kEmptySlot));
        if (lane < R) B.all[lane] = a0;
        if (lane + 32 < R) B.all[lane + 32] = a1;
        if (lane == 0) {
          B.all[R] = v;
          cnt_s = cnt;
          if (cnt < R) row[cnt] = v;
        }
      }
      __syncthreads();
      const bool room = cnt_s < R;
      __syncthreads();  // cnt_s is read by every thread before the next entry rewrites it
      if (room) continue;
      if (tid == 0) atomicAdd(stats + 2, 1ull);
      for (uint32_t idx = tid; idx < n * c4; idx += kRevThreads) {
        const uint32_t r = idx / c4, c = idx - r * c4;
        __pipeline_memcpy_async(rows + size_t(r) * s4 + c, reinterpret_cast<const float4*>(vec_row(ix, B.all[r])) + c,
                                16);
      }
      __pipeline_commit();
      __pipeline_wait_prior(0);
      __syncthreads();
      auto srow = [&](uint32_t r) -> const float* { return reinterpret_cast<const float*>(rows + size_t(r) * s4); };
      // distances to the target (batch_l2_squared_distance_kernel<4> order), two rows per lane quad
      for (uint32_t i0 = 0; i0 < n; i0 += kRevThreads / 2) {
        const uint32_t iA = i0 + (tid >> 2), iB = iA + kRevThreads / 4;
        float pA = 0.f, pB = 0.f;
        if (iA < n) l2_quad2_any(tv, srow(iA), srow(iB < n ? iB : iA), dim, tid & 3, pA, pB);
        const float tA = quad_butterfly(pA), tB = quad_butterfly(pB);
        if ((tid & 3) == 0) {
          if (iA < n) B.d[iA] = tA;
          if (iB < n) B.d[iB] = tB;
        }
      }
      // every pair distance, Dm[a*n + b] = Dm[b*n + a].  The loops run the
      // same trips in every thread (item k found by a scan over all rows,
      // spare threads computing a discarded item), so a warp never splits
      // over the long chains.
      {
        const uint32_t items = item_count(n);
        for (uint32_t k0 = 0; k0 < items; k0 += kRevThreads) {
          const uint32_t k = k0 + tid;
          uint32_t i = 0, base = 0, acc = 0;
          for (uint32_t r = 0; r < n; ++r) {
            const uint32_t q = row_items(n, r);
            if (k >= acc + q) {
              i = r + 1;
              base = acc + q;
            }
            acc += q;
          }
          const bool live = k < items;
          if (!live) i = 0, base = 0;
          const uint32_t Q = row_items(n, i), m = live ? k - base : 0;
          const float* ri = srow(i);
          const float* rj[kRevPartners];
#pragma unroll
          for (int q = 0; q < int(kRevPartners); ++q) {
            const uint32_t j = i + 1 + m + Q * q;
            rj[q] = j < n ? srow(j) : ri;
          }
          float dq[kRevPartners];
          __syncwarp();
          chain_l2_multi<kRevPartners>(ri, rj, dim, dq);
#pragma unroll
          for (int q = 0; q < int(kRevPartners); ++q) {
            const uint32_t j = i + 1 + m + Q * q;
            if (live && j < n) {
              Dm[i * n + j] = dq[q];
              Dm[j * n + i] = dq[q];
            }
          }
        }
      }
      __syncthreads();
      if (tid < 32) {
        for (uint32_t i = lane; i < n; i += 32) {
          const float di = B.d[i];
          uint32_t rk = 0;
          for (uint32_t j = 0; j < n; ++j) rk += (B.d[j] < di) || (B.d[j] == di && j < i);
          B.order[rk] = i;
          B.sd[rk] = di;
          B.valid[rk] = 1;
        }
        __syncwarp();
        uint32_t kept = 0;
        for (uint32_t s = 0; s < n && kept < R; ++s) {
          if (!B.valid[s]) continue;
          const uint32_t ps = B.order[s];
          if (lane == 0) B.kept[kept] = B.all[ps];
          ++kept;
          for (uint32_t i = s + 1 + lane; i < n; i += 32)
            if (B.valid[i] && __fmul_rn(alpha, Dm[ps * n + B.order[i]]) <= B.sd[i]) B.valid[i] = 0;
          __syncwarp();
        }
        for (uint32_t j = lane; j < R; j += 32) row[j] = j < kept ? B.kept[j] : kEmptySlot;
      }
      __syncthreads();
    }
  }
}

// (target, new slot) pairs of the step's new adjacency rows in insert order:
// entry i*R + j is row i's j-th neighbour (empty slots keep the empty key).
__global__ void edge_pairs_kernel(const uint32_t* __restrict__ rows, uint32_t m, uint32_t R, uint32_t n0,
                                  uint32_t* __restrict__ keys, uint32_t* __restrict__ vals) {
  const uint32_t e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= m) return;
  keys[e] = rows[e];
  vals[e] = n0 + e / R;
}

// Sums of the insert searches' counters (H, E) into stats[0], stats[1].
__global__ void sum_counters_kernel(const uint32_t* __restrict__ counters, uint32_t b,
                                    unsigned long long* __restrict__ stats) {
  unsigned long long h = 0, e = 0;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < b; i += gridDim.x * blockDim.x) {
    h += counters[size_t(i) * 4 + 0];
    e += counters[size_t(i) * 4 + 1];
  }
  for (int o = 16; o > 0; o >>= 1) {
    h += __shfl_xor_sync(0xFFFFFFFFu, h, o);
    e += __shfl_xor_sync(0xFFFFFFFFu, e, o);
  }
  if ((threadIdx.x & 31) == 0) {
    atomicAdd(stats + 0, h);
    atomicAdd(stats + 1, e);
  }
}

constexpr uint32_t kInsertDefaultLc = 200;   // --beam-width-construction default (configuration.hh:120)
constexpr float kInsertDefaultAlpha = 1.2f;  // --alpha default (configuration.hh:126)
constexpr uint32_t kInsertDefaultBatch = 1024;

// Scratch of the insert steps, kept on the device between calls (a step
// allocates nothing once it has grown): m = b*R sort keys and values in and
// out, run targets, counts and offsets, the run count, CUB's temp storage, the
// step counters (H, E, full prunes, largest group) and four phase events.
dvs_status ensure_insert_scratch(Device& d, uint32_t m) {
  const size_t words = 7 * size_t(m) + 4;
  if (words > d.ins_buf_words) {
    dev_free(d.ins_buf);
    DVS_CUDA(cudaMalloc(&d.ins_buf, words * 4));
    d.ins_buf_words = words;
  }
  uint32_t* k = d.ins_buf;
  size_t t1 = 0, t2 = 0, t3 = 0;
  DVS_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, t1, k, k, k, k, int(m), 0, 32, d.ins.stream));
  DVS_CUDA(cub::DeviceRunLengthEncode::Encode(nullptr, t2, k, k, k, k, int(m), d.ins.stream));
  DVS_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, t3, k, k, int(m) + 1, d.ins.stream));
  const size_t temp = std::max({t1, t2, t3});
  if (temp > d.ins_temp_bytes) {
    dev_free(d.ins_temp);
    DVS_CUDA(cudaMalloc(&d.ins_temp, temp));
    d.ins_temp_bytes = temp;
  }
  for (auto& e : d.ins_ev)
    if (!e) DVS_CUDA(cudaEventCreate(&e));
  return DVS_OK;
}

// Quantizes rows already rotated in d.ins.qrot (b of them) into records row0..row0+b-1.
dvs_status quantize_rows(Device& d, uint32_t b, uint64_t row0, double tc) {
  const DevLayout& L = d.lay;
  const uint32_t blocks = (b + kQuantPerBlock - 1) / kQuantPerBlock;
  const size_t smem = size_t(kQuantPerBlock) * L.dim;
  if (smem > 48 * 1024)
    DVS_CUDA(cudaFuncSetAttribute(insert_quantize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  insert_quantize_kernel<<<blocks, 32, smem, d.ins.stream>>>(d.ins.qrot, L.vec_stride, L.c_rot, 0.0 + tc, L.dim, L.bits, b,
                                                         d.rec, L.rec_words, L.code_words, row0);
  DVS_CUDA(cudaGetLastError());
  return DVS_OK;
}

// One step of b vectors on one device (all b search the graph of the step's start).
dvs_status insert_step(dvs_index* ix, Device& d, const float* hx, const uint32_t* hid, uint32_t b, uint32_t Lc,
                       float alpha, dvs_insert_stats& st) {
  // only inserts change the layout and they run one at a time: a copy needs
  // no lock; what the step changes is published under the index lock
  DevLayout L = d.lay;
  const uint32_t dim = L.dim, R = L.R;
  const double tc = ix->host.info.t_const;
  const uint64_t n0 = L.n;
  dvs_status r = ensure_scratch(d, d.ins, b, Lc, true);
  if (r == DVS_OK) r = ensure_insert_scratch(d, b * R);
  if (r != DVS_OK) return r;
  DVS_CUDA(cudaMemcpyAsync(d.ins.queries, hx, size_t(b) * dim * 4, cudaMemcpyHostToDevice, d.ins.stream));
  // the vectors, ids and records of the new rows
  DVS_CUDA(cudaMemcpy2DAsync(d.vecs + n0 * L.vec_stride, size_t(L.vec_stride) * 4, d.ins.queries, size_t(dim) * 4,
                             size_t(dim) * 4, b, cudaMemcpyDeviceToDevice, d.ins.stream));
  DVS_CUDA(cudaMemcpyAsync(d.ids + n0, hid, size_t(b) * 4, cudaMemcpyHostToDevice, d.ins.stream));
  DVS_CUDA(launch_prepare(d.ins.queries, dim, L.P, L.c_rot, d.ins.qrot, L.vec_stride, d.ins.qfac, 4, dim, L.bits, b, d.ins.stream));
  r = quantize_rows(d, b, n0, tc);
  if (r != DVS_OK) return r;
  if (n0 == 0) {
    // first node of an empty index: the medoid, no neighbours
    DVS_CUDA(cudaMemsetAsync(d.adj, 0xFF, size_t(R) * 4, d.ins.stream));
    DVS_CUDA(cudaStreamSynchronize(d.ins.stream));
    std::lock_guard<std::mutex> g(ix->mu);
    d.lay.medoid = 0;
    d.lay.n = 1;
    d.rows = 1;
    return DVS_OK;
  }
  // 1. beam search with exact distances, capacity L_c; the whole final beam as slots
  r = search_on(ix, d, d.ins, d.ins.queries, b, Lc, Lc, DVS_MODE_EXACT_GPU, d.ins.out_ids, d.ins.out_dist, d.ins.counters, d.ins.stream, true,
                true);
  if (r != DVS_OK) return r;
  // 3. RobustPrune of each beam into the new adjacency rows
  DVS_CUDA(cudaEventRecord(d.ins_ev[0], d.ins.stream));
  const size_t pstaged = size_t(Lc) * prune_row_stride4(L.vec_stride) * 16 + size_t(Lc) * 9 + 16;
  if (pstaged <= kStageBudget) {
    if (pstaged > 48 * 1024)
      DVS_CUDA(cudaFuncSetAttribute(insert_prune_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(pstaged)));
    insert_prune_kernel<<<b, kPruneThreads, pstaged, d.ins.stream>>>(L, d.ins.out_ids, d.ins.out_dist, d.ins.counters, Lc, alpha, n0,
                                                                 d.adj);
  } else {
    const size_t psmem = prune_passes_bytes(Lc, L.vec_stride);
    if (psmem > 227 * 1024) return fail(DVS_ERR_CAPACITY, "prune pivots need more shared memory than a block has");
    if (psmem > 48 * 1024)
      DVS_CUDA(cudaFuncSetAttribute(insert_prune_passes_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(psmem)));
    insert_prune_passes_kernel<<<b, kPruneThreads, psmem, d.ins.stream>>>(L, d.ins.out_ids, d.ins.out_dist, d.ins.counters, Lc, alpha,
                                                                      n0, d.adj);
  }
  DVS_CUDA(cudaGetLastError());
  DVS_CUDA(cudaEventRecord(d.ins_ev[1], d.ins.stream));
  sum_counters_kernel<<<std::min<uint32_t>((b + 255) / 256, 64), 256, 0, d.ins.stream>>>(d.ins.counters, b, d.ins_stats);
  DVS_CUDA(cudaGetLastError());
  // 5. reverse edges: (target, new slot) pairs grouped by target on the device
  //    with a stable radix sort (insert order kept inside a group)
  const uint32_t m = b * R;
  uint32_t* keys_in = d.ins_buf;
  uint32_t* vals_in = keys_in + m;
  uint32_t* keys_out = vals_in + m;
  uint32_t* vals_out = keys_out + m;
  uint32_t* run_tg = vals_out + m;
  uint32_t* run_cnt = run_tg + m;        // m + 1 entries
  uint32_t* run_off = run_cnt + m + 1;   // m + 1 entries
  uint32_t* nruns = run_off + m + 1;
  DVS_CUDA(cudaEventRecord(d.ins_ev[2], d.ins.stream));
  edge_pairs_kernel<<<(m + 255) / 256, 256, 0, d.ins.stream>>>(d.adj + n0 * R, m, R, uint32_t(n0), keys_in, vals_in);
  DVS_CUDA(cudaGetLastError());
  size_t tb = d.ins_temp_bytes;
  DVS_CUDA(cub::DeviceRadixSort::SortPairs(d.ins_temp, tb, keys_in, keys_out, vals_in, vals_out, int(m), 0, 32,
                                           d.ins.stream));
  tb = d.ins_temp_bytes;
  DVS_CUDA(cub::DeviceRunLengthEncode::Encode(d.ins_temp, tb, keys_out, run_tg, run_cnt, nruns, int(m), d.ins.stream));
  tb = d.ins_temp_bytes;
  DVS_CUDA(cub::DeviceScan::ExclusiveSum(d.ins_temp, tb, run_cnt, run_off, int(m) + 1, d.ins.stream));
  L.n = n0 + b;
  if (rev_warp_bytes(R, L.vec_stride, true) > kRevStageMax && rev_block_bytes(R, L.vec_stride) <= 227 * 1024) {
    // wide rows: a block per target shares one staging
    const size_t smem = rev_block_bytes(R, L.vec_stride);
    DVS_CUDA(cudaFuncSetAttribute(reverse_edges_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(smem)));
    int bps = 0;
    DVS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, reverse_edges_block_kernel, kRevThreads, smem));
    if (bps == 0) return fail(DVS_ERR_CAPACITY, "reverse-edge block needs more shared memory than a block has");
    const uint32_t blocks = std::max(1u, std::min<uint32_t>(m, d.sm_count * uint32_t(bps)));
    reverse_edges_block_kernel<<<blocks, kRevThreads, smem, d.ins.stream>>>(L, d.adj, run_tg, run_off, vals_out, nruns,
                                                                        alpha, d.ins_stats);
  } else {
    // staged when a warp's candidate rows fit kRevStageMax; warps per block
    // chosen for the most resident warps
    const bool staged = rev_warp_bytes(R, L.vec_stride, true) <= kRevStageMax;
    const size_t per_warp = rev_warp_bytes(R, L.vec_stride, staged);
    int best = 0;
    uint32_t wpb = 1, bps = 1;
    for (uint32_t w : {1u, 2u, 4u}) {
      const size_t smem = w * per_warp;
      if (smem > 227 * 1024) break;
      int nb = 0;
      if (staged) {
        DVS_CUDA(cudaFuncSetAttribute(reverse_edges_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(smem)));
        DVS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, reverse_edges_kernel<true>, int(w * 32), smem));
      } else {
        DVS_CUDA(cudaFuncSetAttribute(reverse_edges_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      int(smem)));
        DVS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, reverse_edges_kernel<false>, int(w * 32), smem));
      }
      if (int(w) * nb > best) {
        best = int(w) * nb;
        wpb = w;
        bps = uint32_t(nb);
      }
    }
    if (best == 0) return fail(DVS_ERR_CAPACITY, "reverse-edge warp needs more shared memory than a block has");
    const size_t smem = wpb * per_warp;
    const uint32_t blocks = std::max(1u, std::min<uint32_t>((m + wpb - 1) / wpb, d.sm_count * bps));
    if (staged) {
      DVS_CUDA(cudaFuncSetAttribute(reverse_edges_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(smem)));
      reverse_edges_kernel<true><<<blocks, wpb * 32, smem, d.ins.stream>>>(L, d.adj, run_tg, run_off, vals_out, nruns,
                                                                       alpha, d.ins_stats);
    } else {
      DVS_CUDA(cudaFuncSetAttribute(reverse_edges_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(smem)));
      reverse_edges_kernel<false><<<blocks, wpb * 32, smem, d.ins.stream>>>(L, d.adj, run_tg, run_off, vals_out, nruns,
                                                                        alpha, d.ins_stats);
    }
  }
  DVS_CUDA(cudaGetLastError());
  DVS_CUDA(cudaEventRecord(d.ins_ev[3], d.ins.stream));
  uint32_t work[4] = {0, 0, 0, 0};
  DVS_CUDA(cudaMemcpyAsync(work, d.ins.work, 16, cudaMemcpyDeviceToHost, d.ins.stream));
  DVS_CUDA(cudaStreamSynchronize(d.ins.stream));
  {
    std::lock_guard<std::mutex> g(ix->mu);
    d.lay.n = L.n;
    d.rows = L.n;
  }
  float ms = 0.f;
  DVS_CUDA(cudaEventElapsedTime(&ms, d.ins.ev0, d.ins.ev1));
  st.device_ms += ms;
  DVS_CUDA(cudaEventElapsedTime(&ms, d.ins_ev[0], d.ins_ev[1]));
  st.prune_ms += ms;
  DVS_CUDA(cudaEventElapsedTime(&ms, d.ins_ev[2], d.ins_ev[3]));
  st.reverse_ms += ms;
  if (work[1] & kErrCapacity)
    return fail(DVS_ERR_CAPACITY, "an insert's visited set exceeded its capacity; that vector's links are partial");
  return DVS_OK;
}

}  // namespace

// Grows the device arrays of a replicated index to hold `rows` nodes.
dvs_status grow_rows(Device& d, uint64_t rows) {
  if (rows <= d.cap_rows) return DVS_OK;
  DevLayout& L = d.lay;
  const uint64_t cap = std::max<uint64_t>({rows, d.cap_rows * 2, 1024});
  const uint64_t n = L.n;
  DVS_CUDA(cudaSetDevice(d.ordinal));
  DVS_CUDA(cudaStreamSynchronize(d.ins.stream));
  DVS_CUDA(cudaStreamSynchronize(d.sc.stream));
  uint32_t *adj = nullptr, *rec = nullptr, *ids = nullptr;
  float* vecs = nullptr;
  DVS_CUDA(cudaMalloc(&adj, cap * L.R * 4));
  DVS_CUDA(cudaMalloc(&rec, cap * L.rec_words * 4));
  DVS_CUDA(cudaMalloc(&vecs, cap * L.vec_stride * 4));
  DVS_CUDA(cudaMalloc(&ids, cap * 4));
  DVS_CUDA(cudaMemsetAsync(adj, 0xFF, cap * L.R * 4, d.sc.stream));
  DVS_CUDA(cudaMemsetAsync(rec, 0, cap * L.rec_words * 4, d.sc.stream));
  DVS_CUDA(cudaMemsetAsync(vecs, 0, cap * L.vec_stride * 4, d.sc.stream));
  DVS_CUDA(cudaMemsetAsync(ids, 0, cap * 4, d.sc.stream));
  if (n) {
    DVS_CUDA(cudaMemcpyAsync(adj, d.adj, n * L.R * 4, cudaMemcpyDeviceToDevice, d.sc.stream));
    DVS_CUDA(cudaMemcpyAsync(rec, d.rec, n * L.rec_words * 4, cudaMemcpyDeviceToDevice, d.sc.stream));
    DVS_CUDA(cudaMemcpyAsync(vecs, d.vecs, n * L.vec_stride * 4, cudaMemcpyDeviceToDevice, d.sc.stream));
    DVS_CUDA(cudaMemcpyAsync(ids, d.ids, n * 4, cudaMemcpyDeviceToDevice, d.sc.stream));
  }
  DVS_CUDA(cudaStreamSynchronize(d.sc.stream));
  dev_free(d.adj);
  dev_free(d.rec);
  dev_free(d.vecs);
  dev_free(d.ids);
  d.adj = adj;
  d.rec = rec;
  d.vecs = vecs;
  d.ids = ids;
  L.adj = L.adj_s[0] = adj;
  L.rec = L.rec_s[0] = rec;
  L.vecs = L.vecs_s[0] = vecs;
  L.ids = ids;
  d.cap_rows = cap;
  return DVS_OK;
}

}  // namespace dvs

extern "C" {

dvs_status dvs_reserve(dvs_index* ix, uint64_t capacity) {
  if (!ix) return fail(DVS_ERR_ARG, "null index");
  std::lock_guard<std::mutex> gi(ix->ins_mu);
  std::lock_guard<std::mutex> g(ix->mu);
  for (auto& d : ix->devs) {
    if (d.lay.shard_log != 0) return fail(DVS_ERR_UNSUPPORTED, "online insert needs a replicated index");
    DVS_CUDA(cudaSetDevice(d.ordinal));
    DVS_CUDA(cudaDeviceSynchronize());  // searches in flight on any stream finish first
    const dvs_status s = dvs::grow_rows(d, capacity);
    if (s != DVS_OK) return s;
  }
  return DVS_OK;
}

dvs_status dvs_insert(dvs_index* ix, const float* h_vectors, const uint32_t* h_ids, uint32_t n, uint32_t dim,
                      const dvs_insert_params* p, dvs_insert_stats* stats) {
  if (stats) *stats = dvs_insert_stats{};
  if (!ix) return fail(DVS_ERR_ARG, "null index");
  if (dim != ix->host.info.dim)
    return fail(DVS_ERR_DIM, "insert dimension mismatch: index " + std::to_string(ix->host.info.dim) + ", vector " +
                                 std::to_string(dim));
  if (n == 0) return DVS_OK;
  if (!h_vectors) return fail(DVS_ERR_ARG, "null buffer");
  for (size_t i = 0; i < size_t(n) * dim; ++i)
    if (!std::isfinite(h_vectors[i])) return fail(DVS_ERR_ARG, "vector contains a non-finite value");
  const uint32_t Lc = p && p->beam_width_construction ? p->beam_width_construction : dvs::kInsertDefaultLc;
  const float alpha = p && p->alpha > 0.f ? p->alpha : dvs::kInsertDefaultAlpha;
  const uint32_t max_batch = p && p->max_batch ? p->max_batch : dvs::kInsertDefaultBatch;
  if (Lc > 4096) return fail(DVS_ERR_ARG, "beam_width_construction above 4096 is not supported");
  if (ix->host.info.R > 64) return fail(DVS_ERR_UNSUPPORTED, "max out-degree above 64 is not supported");
  // one insert at a time; searches hold the index lock only to enqueue, and
  // an insert takes it to grow the arrays and to publish each step, so
  // searches run on the GPU while an insert step does
  std::lock_guard<std::mutex> gi(ix->ins_mu);
  uint64_t n_start = 0;
  {
    std::lock_guard<std::mutex> g(ix->mu);
    for (auto& d : ix->devs)
      if (d.lay.shard_log != 0) return fail(DVS_ERR_UNSUPPORTED, "online insert needs a replicated index");
    n_start = ix->devs[0].lay.n;
    if (n_start + n > 0xFFFFFFFEull) return fail(DVS_ERR_CAPACITY, "an index holds at most 2^32 - 2 nodes");
    for (auto& d : ix->devs) {
      if (n_start + n <= d.cap_rows) continue;
      DVS_CUDA(cudaSetDevice(d.ordinal));
      DVS_CUDA(cudaDeviceSynchronize());  // searches in flight on any stream finish before the arrays move
      const dvs_status s = dvs::grow_rows(d, n_start + n);
      if (s != DVS_OK) return s;
    }
  }
  std::vector<uint32_t> ids(n);
  for (uint32_t i = 0; i < n; ++i) ids[i] = h_ids ? h_ids[i] : uint32_t(n_start + i);
  dvs_insert_stats st{};
  for (auto& d : ix->devs) {
    DVS_CUDA(cudaSetDevice(d.ordinal));
    dvs_status s = DVS_OK;
    if (!d.ins_stats) DVS_CUDA(cudaMalloc(&d.ins_stats, 4 * sizeof(unsigned long long)));
    DVS_CUDA(cudaMemsetAsync(d.ins_stats, 0, 4 * sizeof(unsigned long long), d.ins.stream));
    dvs_insert_stats dst{};
    uint32_t pos = 0;
    while (pos < n && s == DVS_OK) {
      const uint64_t cur = d.lay.n;
      const uint32_t b = uint32_t(std::min<uint64_t>({uint64_t(max_batch), std::max<uint64_t>(cur, 1),
                                                      uint64_t(n - pos)}));
      s = dvs::insert_step(ix, d, h_vectors + size_t(pos) * dim, ids.data() + pos, b, Lc, alpha, dst);
      pos += b;
      ++dst.steps;
    }
    if (s != DVS_OK) return s;
    unsigned long long cs[4] = {0, 0, 0, 0};
    DVS_CUDA(cudaMemcpyAsync(cs, d.ins_stats, sizeof(cs), cudaMemcpyDeviceToHost, d.ins.stream));
    DVS_CUDA(cudaStreamSynchronize(d.ins.stream));
    dst.expansions = cs[0];
    dst.distances = cs[1];
    dst.full_prunes = cs[2];
    dst.max_incoming = uint32_t(cs[3]);
    dst.inserted = n;
    if (&d == &ix->devs[0]) st = dst;
  }
  std::lock_guard<std::mutex> g(ix->mu);
  ix->host.info.num_vectors = ix->devs[0].lay.n;
  ix->host.info.medoid = ix->devs[0].lay.medoid;
  if (stats) *stats = st;
  return DVS_OK;
}

}  // extern "C"
