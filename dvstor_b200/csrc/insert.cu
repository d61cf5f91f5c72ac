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
// largest reverse-edge warp that stages its candidate rows (768-dim rows at
// R = 32 still do: two warps per SM reading shared memory beat many warps
// reading each candidate row from L2 at every greedy step)
constexpr size_t kRevStageMax = 120 * 1024;

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
// The kept slots are the new node's adjacency row (row0 + v).  STAGED: the
// candidates' vectors are copied to shared memory once (cp.async, when Lc rows
// fit) at an odd float4 stride, so the greedy loop reads no global memory and
// threads reading consecutive candidates hit distinct banks.
template <bool STAGED>
__global__ void __launch_bounds__(kPruneThreads) insert_prune_kernel(const DevLayout ix, const uint32_t* __restrict__ cand,
                                                                     const float* __restrict__ cand_d,
                                                                     const uint32_t* __restrict__ counters, uint32_t Lc,
                                                                     float alpha, uint64_t row0,
                                                                     uint32_t* __restrict__ adj) {
  extern __shared__ __align__(16) float sm[];
  const uint32_t v = blockIdx.x, tid = threadIdx.x, R = ix.R, dim = ix.dim, vs = ix.vec_stride;
  const uint32_t rs = 4 * prune_row_stride4(vs);             // floats between staged rows
  float* rows = sm;                                          // STAGED: Lc candidate vectors; else p*'s vector
  float* dd = rows + (STAGED ? size_t(Lc) * rs : vs);        // candidate distances
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
  if (STAGED) {
    const uint32_t c4 = vs >> 2;
    for (uint32_t idx = tid; idx < n * c4; idx += blockDim.x) {
      const uint32_t r = idx / c4, c = idx - r * c4;
      __pipeline_memcpy_async(reinterpret_cast<float4*>(rows + size_t(r) * rs) + c,
                              reinterpret_cast<const float4*>(vec_row(ix, sl[r])) + c, 16);
    }
    __pipeline_commit();
    __pipeline_wait_prior(0);
    __syncthreads();
  }
  uint32_t kept = 0;  // identical in every thread
  for (uint32_t s = 0; s < n && kept < R; ++s) {
    if (!valid[s]) continue;
    const uint32_t pslot = sl[s];
    if (tid == 0) row[kept] = pslot;
    ++kept;
    const float* pv = rows + size_t(s) * rs;
    if (!STAGED) {
      const float* g = vec_row(ix, pslot);
      for (uint32_t k = tid; k < dim; k += blockDim.x) rows[k] = g[k];
      pv = rows;
      __syncthreads();
    }
    for (uint32_t i = s + 1 + tid; i < n; i += blockDim.x) {
      if (!valid[i]) continue;
      const float d = chain_l2(pv, STAGED ? rows + size_t(i) * rs : vec_row(ix, sl[i]), dim);
      if (__fmul_rn(alpha, d) <= dd[i]) valid[i] = 0;
    }
    __syncthreads();
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
  DVS_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, t1, k, k, k, k, int(m), 0, 32, d.stream));
  DVS_CUDA(cub::DeviceRunLengthEncode::Encode(nullptr, t2, k, k, k, k, int(m), d.stream));
  DVS_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, t3, k, k, int(m) + 1, d.stream));
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

// Quantizes rows already rotated in d.qrot (b of them) into records row0..row0+b-1.
dvs_status quantize_rows(Device& d, uint32_t b, uint64_t row0, double tc) {
  const DevLayout& L = d.lay;
  const uint32_t blocks = (b + kQuantPerBlock - 1) / kQuantPerBlock;
  const size_t smem = size_t(kQuantPerBlock) * L.dim;
  if (smem > 48 * 1024)
    DVS_CUDA(cudaFuncSetAttribute(insert_quantize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  insert_quantize_kernel<<<blocks, 32, smem, d.stream>>>(d.qrot, L.vec_stride, L.c_rot, 0.0 + tc, L.dim, L.bits, b,
                                                         d.rec, L.rec_words, L.code_words, row0);
  DVS_CUDA(cudaGetLastError());
  return DVS_OK;
}

// One step of b vectors on one device (all b search the graph of the step's start).
dvs_status insert_step(dvs_index* ix, Device& d, const float* hx, const uint32_t* hid, uint32_t b, uint32_t Lc,
                       float alpha, dvs_insert_stats& st) {
  DevLayout& L = d.lay;
  const uint32_t dim = L.dim, R = L.R;
  const double tc = ix->host.info.t_const;
  const uint64_t n0 = L.n;
  dvs_status r = ensure_scratch(d, b, Lc, true);
  if (r == DVS_OK) r = ensure_insert_scratch(d, b * R);
  if (r != DVS_OK) return r;
  DVS_CUDA(cudaMemcpyAsync(d.queries, hx, size_t(b) * dim * 4, cudaMemcpyHostToDevice, d.stream));
  // the vectors, ids and records of the new rows
  DVS_CUDA(cudaMemcpy2DAsync(d.vecs + n0 * L.vec_stride, size_t(L.vec_stride) * 4, d.queries, size_t(dim) * 4,
                             size_t(dim) * 4, b, cudaMemcpyDeviceToDevice, d.stream));
  DVS_CUDA(cudaMemcpyAsync(d.ids + n0, hid, size_t(b) * 4, cudaMemcpyHostToDevice, d.stream));
  DVS_CUDA(launch_prepare(d.queries, dim, L.P, L.c_rot, d.qrot, L.vec_stride, d.qfac, 4, dim, L.bits, b, d.stream));
  r = quantize_rows(d, b, n0, tc);
  if (r != DVS_OK) return r;
  if (n0 == 0) {
    // first node of an empty index: the medoid, no neighbours
    DVS_CUDA(cudaMemsetAsync(d.adj, 0xFF, size_t(R) * 4, d.stream));
    DVS_CUDA(cudaStreamSynchronize(d.stream));
    L.medoid = 0;
    L.n = 1;
    d.rows = 1;
    return DVS_OK;
  }
  // 1. beam search with exact distances, capacity L_c; the whole final beam as slots
  r = search_on(ix, d, d.queries, b, Lc, Lc, DVS_MODE_EXACT_GPU, d.out_ids, d.out_dist, d.counters, d.stream, true,
                true);
  if (r != DVS_OK) return r;
  // 3. RobustPrune of each beam into the new adjacency rows
  DVS_CUDA(cudaEventRecord(d.ins_ev[0], d.stream));
  const size_t pstaged = size_t(Lc) * prune_row_stride4(L.vec_stride) * 16 + size_t(Lc) * 9 + 16;
  if (pstaged <= kStageBudget) {
    if (pstaged > 48 * 1024)
      DVS_CUDA(cudaFuncSetAttribute(insert_prune_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(pstaged)));
    insert_prune_kernel<true><<<b, kPruneThreads, pstaged, d.stream>>>(L, d.out_ids, d.out_dist, d.counters, Lc, alpha,
                                                                       n0, d.adj);
  } else {
    const size_t psmem = size_t(L.vec_stride) * 4 + size_t(Lc) * 9 + 16;
    if (psmem > 48 * 1024)
      DVS_CUDA(cudaFuncSetAttribute(insert_prune_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(psmem)));
    insert_prune_kernel<false><<<b, kPruneThreads, psmem, d.stream>>>(L, d.out_ids, d.out_dist, d.counters, Lc, alpha,
                                                                      n0, d.adj);
  }
  DVS_CUDA(cudaGetLastError());
  DVS_CUDA(cudaEventRecord(d.ins_ev[1], d.stream));
  sum_counters_kernel<<<std::min<uint32_t>((b + 255) / 256, 64), 256, 0, d.stream>>>(d.counters, b, d.ins_stats);
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
  DVS_CUDA(cudaEventRecord(d.ins_ev[2], d.stream));
  edge_pairs_kernel<<<(m + 255) / 256, 256, 0, d.stream>>>(d.adj + n0 * R, m, R, uint32_t(n0), keys_in, vals_in);
  DVS_CUDA(cudaGetLastError());
  size_t tb = d.ins_temp_bytes;
  DVS_CUDA(cub::DeviceRadixSort::SortPairs(d.ins_temp, tb, keys_in, keys_out, vals_in, vals_out, int(m), 0, 32,
                                           d.stream));
  tb = d.ins_temp_bytes;
  DVS_CUDA(cub::DeviceRunLengthEncode::Encode(d.ins_temp, tb, keys_out, run_tg, run_cnt, nruns, int(m), d.stream));
  tb = d.ins_temp_bytes;
  DVS_CUDA(cub::DeviceScan::ExclusiveSum(d.ins_temp, tb, run_cnt, run_off, int(m) + 1, d.stream));
  L.n = n0 + b;
  {
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
      reverse_edges_kernel<true><<<blocks, wpb * 32, smem, d.stream>>>(L, d.adj, run_tg, run_off, vals_out, nruns,
                                                                       alpha, d.ins_stats);
    } else {
      DVS_CUDA(cudaFuncSetAttribute(reverse_edges_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(smem)));
      reverse_edges_kernel<false><<<blocks, wpb * 32, smem, d.stream>>>(L, d.adj, run_tg, run_off, vals_out, nruns,
                                                                        alpha, d.ins_stats);
    }
  }
  DVS_CUDA(cudaGetLastError());
  DVS_CUDA(cudaEventRecord(d.ins_ev[3], d.stream));
  uint32_t work[4] = {0, 0, 0, 0};
  DVS_CUDA(cudaMemcpyAsync(work, d.work, 16, cudaMemcpyDeviceToHost, d.stream));
  DVS_CUDA(cudaStreamSynchronize(d.stream));
  d.rows = L.n;
  float ms = 0.f;
  DVS_CUDA(cudaEventElapsedTime(&ms, d.ev0, d.ev1));
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
  DVS_CUDA(cudaStreamSynchronize(d.stream));
  uint32_t *adj = nullptr, *rec = nullptr, *ids = nullptr;
  float* vecs = nullptr;
  DVS_CUDA(cudaMalloc(&adj, cap * L.R * 4));
  DVS_CUDA(cudaMalloc(&rec, cap * L.rec_words * 4));
  DVS_CUDA(cudaMalloc(&vecs, cap * L.vec_stride * 4));
  DVS_CUDA(cudaMalloc(&ids, cap * 4));
  DVS_CUDA(cudaMemsetAsync(adj, 0xFF, cap * L.R * 4, d.stream));
  DVS_CUDA(cudaMemsetAsync(rec, 0, cap * L.rec_words * 4, d.stream));
  DVS_CUDA(cudaMemsetAsync(vecs, 0, cap * L.vec_stride * 4, d.stream));
  DVS_CUDA(cudaMemsetAsync(ids, 0, cap * 4, d.stream));
  if (n) {
    DVS_CUDA(cudaMemcpyAsync(adj, d.adj, n * L.R * 4, cudaMemcpyDeviceToDevice, d.stream));
    DVS_CUDA(cudaMemcpyAsync(rec, d.rec, n * L.rec_words * 4, cudaMemcpyDeviceToDevice, d.stream));
    DVS_CUDA(cudaMemcpyAsync(vecs, d.vecs, n * L.vec_stride * 4, cudaMemcpyDeviceToDevice, d.stream));
    DVS_CUDA(cudaMemcpyAsync(ids, d.ids, n * 4, cudaMemcpyDeviceToDevice, d.stream));
  }
  DVS_CUDA(cudaStreamSynchronize(d.stream));
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
  std::lock_guard<std::mutex> g(ix->mu);
  for (auto& d : ix->devs) {
    if (d.lay.shard_log != 0) return fail(DVS_ERR_UNSUPPORTED, "online insert needs a replicated index");
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
  std::lock_guard<std::mutex> g(ix->mu);
  for (auto& d : ix->devs)
    if (d.lay.shard_log != 0) return fail(DVS_ERR_UNSUPPORTED, "online insert needs a replicated index");
  const uint64_t n_start = ix->devs[0].lay.n;
  if (n_start + n > 0xFFFFFFFEull) return fail(DVS_ERR_CAPACITY, "an index holds at most 2^32 - 2 nodes");
  std::vector<uint32_t> ids(n);
  for (uint32_t i = 0; i < n; ++i) ids[i] = h_ids ? h_ids[i] : uint32_t(n_start + i);
  dvs_insert_stats st{};
  for (auto& d : ix->devs) {
    DVS_CUDA(cudaSetDevice(d.ordinal));
    DVS_CUDA(cudaDeviceSynchronize());  // searches in flight on any stream finish first
    dvs_status s = dvs::grow_rows(d, n_start + n);
    if (s != DVS_OK) return s;
    if (!d.ins_stats) DVS_CUDA(cudaMalloc(&d.ins_stats, 4 * sizeof(unsigned long long)));
    DVS_CUDA(cudaMemsetAsync(d.ins_stats, 0, 4 * sizeof(unsigned long long), d.stream));
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
    DVS_CUDA(cudaMemcpyAsync(cs, d.ins_stats, sizeof(cs), cudaMemcpyDeviceToHost, d.stream));
    DVS_CUDA(cudaStreamSynchronize(d.stream));
    dst.expansions = cs[0];
    dst.distances = cs[1];
    dst.full_prunes = cs[2];
    dst.max_incoming = uint32_t(cs[3]);
    dst.inserted = n;
    if (&d == &ix->devs[0]) st = dst;
  }
  ix->host.info.num_vectors = ix->devs[0].lay.n;
  ix->host.info.medoid = ix->devs[0].lay.medoid;
  if (stats) *stats = st;
  return DVS_OK;
}

}  // extern "C"
